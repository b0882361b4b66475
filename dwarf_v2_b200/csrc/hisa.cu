// V16/V18 HISA L3 mixer: chunk representatives, strict-causal top-k tile
// router, and the fused routed + local tile attention.
//
// Replaces, for head_dim 64, chunk 64, selector tile 16, local window 64 and
// enumerate_all token selection (the production configuration):
//   _completed_chunk_representatives (kernels/hierarchical_sparse_attn_v18_hisa.py:171-219)
//   anchor logits + _eligibility + _build_causal_tile_metadata (:2614-2624, 222-237, 290-397)
//   _selected_route_scores (:418-468)
//   FlexAttention local lane (:2424-2461) + _global_lane_forward_kernel (:1002-1100)
//   + _merge_attention_lanes (:808-835)
// The two attention lanes and their exact LSE merge are one softmax over the
// union of the lanes' keys, which is what the fused kernel computes.
//
// Router arithmetic is float32 with fixed left-to-right sums and no FMA
// contraction, so selected chunk indices are reproducible bit for bit by a
// CPU restatement; ties go to the lower chunk index.
#include "common.cuh"

namespace dwarf {
namespace {

constexpr int kHD = 64;
constexpr int kChunk = 64;
constexpr int kTile = 16;
constexpr int kWindow = 64;
constexpr int kTopK = 4;
constexpr int kMaxChunks = 128;
constexpr float kLog2e = 1.4426950408889634f;

__host__ __device__ __forceinline__ int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }

// ---------------------------------------------------------------- representatives

struct RepsParams {
  const __nv_bfloat16* k; int64_t skb, skh, skn;
  const int32_t* lengths;
  __nv_bfloat16* reps;  // [B,H,C,64] contiguous
  int64_t H, T, C;
  float alpha;
};

// One CTA (64 threads) per (chunk, head, batch).
__global__ void __launch_bounds__(64) hisa_reps_kernel(const RepsParams p) {
  __shared__ float xs[kChunk][kHD + 1];
  __shared__ float energy[kChunk];
  __shared__ float rep[kHD];
  __shared__ int best_row;
  __shared__ float norm;
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x;
  const int64_t vlen = imin64((int64_t)p.lengths[b], p.T);
  const __nv_bfloat16* base = p.k + b * p.skb + h * p.skh;
  for (int i = tid; i < kChunk * kHD; i += 64) {
    const int r = i / kHD, d = i % kHD;
    const int64_t t = (int64_t)c * kChunk + r;
    xs[r][d] = t < p.T ? __bfloat162float(base[t * p.skn + d]) : 0.0f;
  }
  __syncthreads();
  // Row energies (row = tid), masked to -inf past the valid length.
  {
    float e = 0.0f;
    for (int d = 0; d < kHD; ++d) e = add_rn(e, mul_rn(xs[tid][d], xs[tid][d]));
    energy[tid] = ((int64_t)c * kChunk + tid < vlen) ? e : -INFINITY;
  }
  __syncthreads();
  if (tid == 0) {
    int bi = 0;
    float bv = energy[0];
    for (int r = 1; r < kChunk; ++r)
      if (energy[r] > bv) { bv = energy[r]; bi = r; }  // first maximum wins
    best_row = bi;
  }
  __syncthreads();
  // Masked mean of dim d (= tid) and the blend.
  {
    float s = 0.0f;
    int count = 0;
    for (int r = 0; r < kChunk; ++r) {
      const bool ok = (int64_t)c * kChunk + r < vlen;
      s = add_rn(s, ok ? xs[r][tid] : 0.0f);
      count += ok;
    }
    const float mean = __fdiv_rn(s, (float)max(count, 1));
    rep[tid] = add_rn(mul_rn(1.0f - p.alpha, mean), mul_rn(p.alpha, xs[best_row][tid]));
  }
  __syncthreads();
  if (tid == 0) {
    float ss = 0.0f;
    for (int d = 0; d < kHD; ++d) ss = add_rn(ss, mul_rn(rep[d], rep[d]));
    norm = fmaxf(sqrtf(ss), 1e-6f);
  }
  __syncthreads();
  const bool chunk_valid = (int64_t)c * kChunk < vlen;
  const float v = chunk_valid ? __fdiv_rn(rep[tid], norm) : 0.0f;
  p.reps[((b * p.H + h) * p.C + c) * kHD + tid] = __float2bfloat16_rn(v);
}

// ---------------------------------------------------------------- router

struct SelectParams {
  const __nv_bfloat16* q; int64_t sqb, sqh, sqn;
  const __nv_bfloat16* reps;  // [B,H,C,64]
  const int32_t* lengths;
  int32_t* top;               // [B,H,tiles,K]
  float* logits;              // optional [B,H,tiles,C], masked (-inf)
  int64_t H, T, C, tiles;
  int k_slots;
  float temperature;
};

// L2-normalise a 64-value row in place: float32 sequential norm, IEEE
// divide, bf16 rounding (F.normalize(x.float(), eps=1e-6).to(bf16)).
__device__ __forceinline__ void normalize_row_bf16(float* row) {
  float ss = 0.0f;
  for (int d = 0; d < kHD; ++d) ss = add_rn(ss, mul_rn(row[d], row[d]));
  const float nrm = fmaxf(sqrtf(ss), 1e-6f);
  for (int d = 0; d < kHD; ++d) row[d] = round_bf16(__fdiv_rn(row[d], nrm));
}

// One warp per selector tile; the CTA's (b, h) representatives sit in smem.
__global__ void __launch_bounds__(256) hisa_select_kernel(const SelectParams p) {
  __shared__ float reps[kMaxChunks][kHD + 1];
  __shared__ float anchor[8][kHD];
  const int h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < p.C * kHD; i += blockDim.x)
    reps[i / kHD][i % kHD] = __bfloat162float(p.reps[((b * p.H + h) * p.C) * kHD + i]);
  const int64_t t = (int64_t)blockIdx.x * 8 + warp;
  const int64_t start = t * kTile;
  const int64_t arow = imin64(start, p.T - 1);
  const __nv_bfloat16* qrow = p.q + b * p.sqb + h * p.sqh + arow * p.sqn;
  anchor[warp][lane] = __bfloat162float(qrow[lane]);
  anchor[warp][lane + 32] = __bfloat162float(qrow[lane + 32]);
  __syncthreads();
  if (t >= p.tiles) return;
  if (lane == 0) normalize_row_bf16(anchor[warp]);
  __syncwarp();
  const int64_t vlen = p.lengths[b];
  float val[kMaxChunks / 32];
#pragma unroll
  for (int i = 0; i < kMaxChunks / 32; ++i) {
    const int c = lane + 32 * i;
    float s = -INFINITY;
    if (c < p.C) {
      float acc = 0.0f;
      for (int d = 0; d < kHD; ++d) acc = add_rn(acc, mul_rn(anchor[warp][d], reps[c][d]));
      acc = __fdiv_rn(acc, p.temperature);
      const bool eligible = ((int64_t)(c + 1) * kChunk <= start) && ((int64_t)c * kChunk < vlen) && (start < vlen);
      s = eligible ? acc : -INFINITY;
      if (p.logits) p.logits[((b * p.H + h) * p.tiles + t) * p.C + c] = s;
    }
    val[i] = s;
  }
  // k rounds of warp argmax: larger value first, lower index on ties.
  int32_t* out = p.top + ((b * p.H + h) * p.tiles + t) * p.k_slots;
  for (int k = 0; k < p.k_slots; ++k) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxChunks / 32; ++i) {
      const int c = lane + 32 * i;
      if (c < p.C && !isnan(val[i]) && (val[i] > bv || (val[i] == bv && c < bi))) { bv = val[i]; bi = c; }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) out[k] = (bi != 0x7fffffff && isfinite(bv)) ? bi : -1;
    // retire the winner (NaN marks "taken")
#pragma unroll
    for (int i = 0; i < kMaxChunks / 32; ++i)
      if (lane + 32 * i == bi) val[i] = NAN;
  }
}

// ---------------------------------------------------------------- tile attention

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}

// Swizzled [rows][64 bf16] tile: 16-byte chunk c of row r lives at chunk c ^ (r & 7).
__device__ __forceinline__ uint32_t tile_addr(uint32_t base, int row, int chunk) {
  return base + row * 128 + ((chunk ^ (row & 7)) << 4);
}

struct AttnParams {
  const __nv_bfloat16* q; int64_t sqb, sqh, sqn;
  const __nv_bfloat16* lk; int64_t slkb, slkh, slkn;
  const __nv_bfloat16* lv; int64_t slvb, slvh, slvn;
  const __nv_bfloat16* gk; int64_t sgkb, sgkh, sgkn;
  const __nv_bfloat16* gv; int64_t sgvb, sgvh, sgvn;
  const __nv_bfloat16* reps;  // [B,H,C,64]
  const int32_t* top;         // [B,H,tiles,K]
  const float* route_scale;   // [H]
  const int32_t* lengths;
  __nv_bfloat16* out; int64_t sob, soh, son;
  __nv_bfloat16* route_out;   // optional [B,H,T,4]
  int64_t H, T, C, tiles;
  int k_slots;
};

constexpr int kAttnWarps = 4;
constexpr int kWarpSmem = 2 * 64 * 128 + 16 * 128 + 16 * kHD * 4 + kTopK * kHD * 4 + 16 * kTopK * 4;

// Stage rows [row0, row0+nrows) of a [T,64] bf16 matrix into a swizzled tile
// (rows outside [0, T) are zero-filled).
__device__ __forceinline__ void stage_rows(uint32_t tile, const __nv_bfloat16* base, int64_t stride, int64_t row0,
                                           int nrows, int64_t T, int lane) {
  for (int i = lane; i < nrows * 8; i += 32) {
    const int r = i >> 3, c = i & 7;
    const int64_t row = row0 + r;
    const bool ok = row >= 0 && row < T;
    cp_async16(tile_addr(tile, r, c), base + (ok ? row : 0) * stride + c * 8, ok);
  }
}

// S[16 x 8*NT] = Q tile . K block^T, online-softmax update, O += P . V.
// Key i of the block is valid for query row r when mask(r, i) holds; bias[rr]
// is added to the scaled score of row g + 8 rr (the route prior of the slot).
template <int NT, typename Mask>
__device__ __forceinline__ void attend_block(const uint32_t (&qa)[4][4], uint32_t ktile, uint32_t vtile,
                                             const float (&bias)[2], Mask mask, float (&o)[8][4], float (&m)[2],
                                             float (&l)[2], int lane) {
  const int g = lane >> 2, t4 = lane & 3;
  float s[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
  for (int kt = 0; kt < 4; ++kt) {
#pragma unroll
    for (int j = 0; j < NT; j += 2) {
      const int mtx = lane >> 3, r = lane & 7;
      const int key = j * 8 + (mtx >> 1) * 8 + r;
      const int chunk = kt * 2 + (mtx & 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4(tile_addr(ktile, key, chunk), b0, b1, b2, b3);
      mma_bf16(s[j], qa[kt], b0, b1);
      if (j + 1 < NT) mma_bf16(s[j + 1], qa[kt], b2, b3);
    }
  }
  float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
  for (int j = 0; j < NT; ++j) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int row = g + (e >> 1) * 8;
      const int key = j * 8 + 2 * t4 + (e & 1);
      const float v = mask(row, key) ? (s[j][e] * 0.125f + bias[e >> 1]) * kLog2e : -INFINITY;
      s[j][e] = v;
      mx[e >> 1] = fmaxf(mx[e >> 1], v);
    }
  }
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 1));
    mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 2));
  }
  float scale[2], msafe[2];
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const float mn = fmaxf(m[rr], mx[rr]);
    msafe[rr] = mn == -INFINITY ? 0.0f : mn;
    scale[rr] = exp2f(m[rr] - msafe[rr]);
    m[rr] = mn;
  }
  float rs[2] = {0.0f, 0.0f};
  uint32_t pa[NT][2];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const float p0 = exp2f(s[j][0] - msafe[0]), p1 = exp2f(s[j][1] - msafe[0]);
    const float p2 = exp2f(s[j][2] - msafe[1]), p3 = exp2f(s[j][3] - msafe[1]);
    rs[0] += p0 + p1;
    rs[1] += p2 + p3;
    pa[j][0] = pack_bf16(p0, p1);
    pa[j][1] = pack_bf16(p2, p3);
  }
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    rs[rr] += __shfl_xor_sync(0xffffffffu, rs[rr], 1);
    rs[rr] += __shfl_xor_sync(0xffffffffu, rs[rr], 2);
    l[rr] = l[rr] * scale[rr] + rs[rr];
  }
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    o[n][0] *= scale[0]; o[n][1] *= scale[0];
    o[n][2] *= scale[1]; o[n][3] *= scale[1];
  }
  // O += P . V over NT/2 key slices of 16 (P from the S accumulators, bf16)
#pragma unroll
  for (int kk = 0; kk < NT / 2; ++kk) {
    const uint32_t a[4] = {pa[2 * kk][0], pa[2 * kk][1], pa[2 * kk + 1][0], pa[2 * kk + 1][1]};
#pragma unroll
    for (int n = 0; n < 8; n += 2) {
      const int mtx = lane >> 3, r = lane & 7;
      const int key = kk * 16 + (mtx & 1) * 8 + r;
      const int chunk = n + (mtx >> 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(tile_addr(vtile, key, chunk), b0, b1, b2, b3);
      mma_bf16(o[n], a, b0, b1);
      mma_bf16(o[n + 1], a, b2, b3);
    }
  }
}

// One warp per 16-query selector tile, 4 tiles of one (b, h) per CTA; each
// warp owns its shared-memory slice and synchronises only itself.
__global__ void __launch_bounds__(kAttnWarps * 32) hisa_attn_kernel(const AttnParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, b = blockIdx.z;
  const int64_t t = (int64_t)blockIdx.x * kAttnWarps + warp;
  if (t >= p.tiles) return;
  unsigned char* ws = smem + warp * kWarpSmem;
  const uint32_t ktile = smem_u32(ws);
  const uint32_t vtile = ktile + 64 * 128;
  __nv_bfloat16* qtile = reinterpret_cast<__nv_bfloat16*>(ws + 2 * 64 * 128);
  float* qhat = reinterpret_cast<float*>(ws + 2 * 64 * 128 + 16 * 128);  // [16][64]
  float* rsel = qhat + 16 * kHD;                                          // [4][64]
  float* route = rsel + kTopK * kHD;                                      // [16][4]
  const int g = lane >> 2, t4 = lane & 3;
  const int64_t t0 = t * kTile;
  const int64_t vlen = imin64((int64_t)p.lengths[b], p.T);

  const __nv_bfloat16* qb = p.q + b * p.sqb + h * p.sqh;
  for (int i = lane; i < 16 * 8; i += 32) {
    const int r = i >> 3, c = i & 7;
    const int64_t row = t0 + r;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < p.T) v = *reinterpret_cast<const uint4*>(qb + row * p.sqn + c * 8);
    *reinterpret_cast<uint4*>(qtile + r * 64 + c * 8) = v;
  }
  int chunk_sel[kTopK];
  const int32_t* top = p.top + ((b * p.H + h) * p.tiles + t) * p.k_slots;
#pragma unroll
  for (int k = 0; k < kTopK; ++k) chunk_sel[k] = k < p.k_slots ? top[k] : -1;
  for (int i = lane; i < kTopK * kHD; i += 32) {
    const int k = i / kHD, d = i % kHD;
    rsel[i] = chunk_sel[k] >= 0 ? __bfloat162float(p.reps[((b * p.H + h) * p.C + chunk_sel[k]) * kHD + d]) : 0.0f;
  }
  __syncwarp();
  // q^ = bf16(q / max(|q|, 1e-6)) for the 16 rows (lanes 0..15 own one row each).
  if (lane < 16) {
    float* row = qhat + lane * kHD;
    for (int d = 0; d < kHD; ++d) row[d] = __bfloat162float(qtile[lane * 64 + d]);
    normalize_row_bf16(row);
  }
  __syncwarp();
  // Route prior: lane -> (row = lane & 15, slots 2*(lane>>4) + {0,1}).
  {
    const int row = lane & 15, k0 = (lane >> 4) * 2;
    float sc[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float acc = 0.0f;
      for (int d = 0; d < kHD; ++d) acc = add_rn(acc, mul_rn(qhat[row * kHD + d], rsel[(k0 + e) * kHD + d]));
      sc[e] = acc;
    }
    const float o0 = __shfl_xor_sync(0xffffffffu, sc[0], 16);
    const float o1 = __shfl_xor_sync(0xffffffffu, sc[1], 16);
    float all[4];
    if (k0 == 0) { all[0] = sc[0]; all[1] = sc[1]; all[2] = o0; all[3] = o1; }
    else { all[0] = o0; all[1] = o1; all[2] = sc[0]; all[3] = sc[1]; }
    float sum = 0.0f;
    int count = 0;
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
      const bool ok = chunk_sel[k] >= 0;
      sum = add_rn(sum, ok ? all[k] : 0.0f);
      count += ok;
    }
    const float mean = __fdiv_rn(sum, (float)max(count, 1));
    const float scale = p.route_scale[h];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int k = k0 + e;
      const float centered = chunk_sel[k] >= 0 ? __fsub_rn(sc[e], mean) : 0.0f;
      const float v = round_bf16(mul_rn(centered, scale));
      route[row * kTopK + k] = v;
      if (p.route_out != nullptr && t0 + row < p.T)
        p.route_out[((b * p.H + h) * p.T + t0 + row) * kTopK + k] = __float2bfloat16_rn(v);
    }
  }
  __syncwarp();
  uint32_t qa[4][4];
#pragma unroll
  for (int kt = 0; kt < 4; ++kt) {
    const int c0 = kt * 16 + 2 * t4;
    qa[kt][0] = *reinterpret_cast<const uint32_t*>(qtile + g * 64 + c0);
    qa[kt][1] = *reinterpret_cast<const uint32_t*>(qtile + (g + 8) * 64 + c0);
    qa[kt][2] = *reinterpret_cast<const uint32_t*>(qtile + g * 64 + c0 + 8);
    qa[kt][3] = *reinterpret_cast<const uint32_t*>(qtile + (g + 8) * 64 + c0 + 8);
  }

  float o[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};
  const float zero_bias[2] = {0.0f, 0.0f};
  const __nv_bfloat16* lkb = p.lk + b * p.slkb + h * p.slkh;
  const __nv_bfloat16* lvb = p.lv + b * p.slvb + h * p.slvh;
  const __nv_bfloat16* gkb = p.gk + b * p.sgkb + h * p.sgkh;
  const __nv_bfloat16* gvb = p.gv + b * p.sgvb + h * p.sgvh;

  // Local window, part 1: rows [t0-64, t0); key i serves query r when i >= r.
  if (t0 > 0) {
    stage_rows(ktile, lkb, p.slkn, t0 - 64, 64, p.T, lane);
    stage_rows(vtile, lvb, p.slvn, t0 - 64, 64, p.T, lane);
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
    __syncwarp();
    auto mask = [&](int r, int i) {
      const int64_t id = t0 - 64 + i;
      return id >= 0 && i >= r && id < vlen && t0 + r < vlen;
    };
    attend_block<8>(qa, ktile, vtile, zero_bias, mask, o, m, l, lane);
    __syncwarp();
  }
  // Local window, part 2: rows [t0, t0+16); strictly earlier rows of the tile.
  {
    stage_rows(ktile, lkb, p.slkn, t0, 16, p.T, lane);
    stage_rows(vtile, lvb, p.slvn, t0, 16, p.T, lane);
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
    __syncwarp();
    auto mask = [&](int r, int i) { return i < r && t0 + i < vlen && t0 + r < vlen; };
    attend_block<2>(qa, ktile, vtile, zero_bias, mask, o, m, l, lane);
    __syncwarp();
  }
  // Routed chunks: ids < n - 64, route prior of the slot added.
#pragma unroll 1
  for (int k = 0; k < kTopK; ++k) {
    const int c = chunk_sel[k];
    if (c < 0) continue;
    const int64_t row0 = (int64_t)c * kChunk;
    stage_rows(ktile, gkb, p.sgkn, row0, 64, p.T, lane);
    stage_rows(vtile, gvb, p.sgvn, row0, 64, p.T, lane);
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
    __syncwarp();
    const float bias[2] = {route[g * kTopK + k], route[(g + 8) * kTopK + k]};
    auto mask = [&](int r, int i) {
      const int64_t id = row0 + i;
      const int64_t n = t0 + r;
      return id < n - kWindow && id < vlen && n < vlen;
    };
    attend_block<8>(qa, ktile, vtile, bias, mask, o, m, l, lane);
    __syncwarp();
  }

  // Epilogue: O / l in bf16; rows past the valid length are zero.
  __nv_bfloat16* ob = p.out + b * p.sob + h * p.soh;
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int64_t row = t0 + g + rr * 8;
    if (row >= p.T) continue;
    const float inv = (l[rr] > 0.0f && row < vlen) ? 1.0f / l[rr] : 0.0f;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const uint32_t v = pack_bf16(o[n][rr * 2] * inv, o[n][rr * 2 + 1] * inv);
      *reinterpret_cast<uint32_t*>(ob + row * p.son + n * 8 + 2 * t4) = v;
    }
  }
}

bool al16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace
}  // namespace dwarf

using namespace dwarf;

extern "C" int dwarf_hisa_reps(const dwarf_hisa_reps_args* a, void* stream) {
  DWARF_CHECK_VERSION(a);
  if (a->head_dim != kHD || a->chunk_size != kChunk) return DWARF_ERR_SHAPE;
  if (a->B < 0 || a->H <= 0 || a->T < 0) return DWARF_ERR_SHAPE;
  if (a->B == 0 || a->T == 0) return DWARF_OK;
  if (!a->key || !a->lengths || !a->reps) return DWARF_ERR_NULL;
  if (!(a->blend_alpha >= 0.0f && a->blend_alpha <= 1.0f)) return DWARF_ERR_VALUE;
  RepsParams p{(const __nv_bfloat16*)a->key, a->skb, a->skh, a->skn, a->lengths, (__nv_bfloat16*)a->reps,
               a->H, a->T, (a->T + kChunk - 1) / kChunk, a->blend_alpha};
  dim3 grid((unsigned)p.C, (unsigned)a->H, (unsigned)a->B);
  hisa_reps_kernel<<<grid, 64, 0, (cudaStream_t)stream>>>(p);
  return launch_status();
}

extern "C" int dwarf_hisa_select(const dwarf_hisa_select_args* a, void* stream) {
  DWARF_CHECK_VERSION(a);
  if (a->head_dim != kHD || a->chunk_size != kChunk || a->selector_tile != kTile) return DWARF_ERR_SHAPE;
  if (a->B < 0 || a->H <= 0 || a->T < 0 || a->top_k < 1) return DWARF_ERR_SHAPE;
  if (a->B == 0 || a->T == 0) return DWARF_OK;
  const int64_t C = (a->T + kChunk - 1) / kChunk;
  if (C > kMaxChunks) return DWARF_ERR_SHAPE;
  if (!a->query || !a->reps || !a->lengths || !a->top_chunk_idx) return DWARF_ERR_NULL;
  if (!(a->temperature > 0.0f)) return DWARF_ERR_VALUE;
  SelectParams p{};
  p.q = (const __nv_bfloat16*)a->query; p.sqb = a->sqb; p.sqh = a->sqh; p.sqn = a->sqn;
  p.reps = (const __nv_bfloat16*)a->reps; p.lengths = a->lengths; p.top = a->top_chunk_idx;
  p.logits = a->logits; p.H = a->H; p.T = a->T; p.C = C; p.tiles = (a->T + kTile - 1) / kTile;
  p.k_slots = (int)(a->top_k < C ? a->top_k : C);
  p.temperature = a->temperature;
  dim3 grid((unsigned)((p.tiles + 7) / 8), (unsigned)a->H, (unsigned)a->B);
  hisa_select_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(p);
  return launch_status();
}

extern "C" int dwarf_hisa_attn(const dwarf_hisa_attn_args* a, void* stream) {
  DWARF_CHECK_VERSION(a);
  if (a->head_dim != kHD || a->chunk_size != kChunk || a->selector_tile != kTile || a->local_window != kWindow)
    return DWARF_ERR_SHAPE;
  if (a->B < 0 || a->H <= 0 || a->T < 0 || a->k_slots < 0 || a->k_slots > kTopK) return DWARF_ERR_SHAPE;
  if (a->B == 0 || a->T == 0) return DWARF_OK;
  if (!a->query || !a->local_key || !a->local_value || !a->global_key || !a->global_value || !a->reps ||
      !a->top_chunk_idx || !a->route_scale || !a->lengths || !a->out)
    return DWARF_ERR_NULL;
  const void* rows[] = {a->query, a->local_key, a->local_value, a->global_key, a->global_value, a->out};
  for (const void* r : rows)
    if (!al16(r)) return DWARF_ERR_ALIGN;
  const int64_t strides[] = {a->sqb, a->sqh, a->sqn, a->slkb, a->slkh, a->slkn, a->slvb, a->slvh, a->slvn,
                             a->sgkb, a->sgkh, a->sgkn, a->sgvb, a->sgvh, a->sgvn, a->sob, a->soh, a->son};
  for (int64_t s : strides)
    if (s % 8 != 0) return DWARF_ERR_ALIGN;
  AttnParams p{};
  p.q = (const __nv_bfloat16*)a->query; p.sqb = a->sqb; p.sqh = a->sqh; p.sqn = a->sqn;
  p.lk = (const __nv_bfloat16*)a->local_key; p.slkb = a->slkb; p.slkh = a->slkh; p.slkn = a->slkn;
  p.lv = (const __nv_bfloat16*)a->local_value; p.slvb = a->slvb; p.slvh = a->slvh; p.slvn = a->slvn;
  p.gk = (const __nv_bfloat16*)a->global_key; p.sgkb = a->sgkb; p.sgkh = a->sgkh; p.sgkn = a->sgkn;
  p.gv = (const __nv_bfloat16*)a->global_value; p.sgvb = a->sgvb; p.sgvh = a->sgvh; p.sgvn = a->sgvn;
  p.reps = (const __nv_bfloat16*)a->reps; p.top = a->top_chunk_idx; p.route_scale = a->route_scale;
  p.lengths = a->lengths;
  p.out = (__nv_bfloat16*)a->out; p.sob = a->sob; p.soh = a->soh; p.son = a->son;
  p.route_out = (__nv_bfloat16*)a->route_out;
  p.H = a->H; p.T = a->T; p.C = (a->T + kChunk - 1) / kChunk; p.tiles = (a->T + kTile - 1) / kTile;
  p.k_slots = a->k_slots;
  const size_t smem = (size_t)kAttnWarps * kWarpSmem;
  if (cudaFuncSetAttribute(hisa_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return DWARF_ERR_LAUNCH;
  dim3 grid((unsigned)((p.tiles + kAttnWarps - 1) / kAttnWarps), (unsigned)a->H, (unsigned)a->B);
  hisa_attn_kernel<<<grid, kAttnWarps * 32, smem, (cudaStream_t)stream>>>(p);
  return launch_status();
}
