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
#include "tma.cuh"

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
  const int64_t* pos;   // optional: only chunk *pos / 64 (decode step)
};

// One CTA (64 threads) per (chunk, head, batch). Operations and summation
// orders are those of the reference; only the serial steps are spread out:
// the chunk arrives by 16-byte loads (8 threads per 128-byte row) when rows are
// aligned, the first-maximum row comes from a shuffle reduction (ties to the
// lower row, as the sequential scan), and the representative's squares are
// formed in parallel and summed in dimension order by every thread.
__global__ void __launch_bounds__(64) hisa_reps_kernel(const RepsParams p) {
  __shared__ float xs[kChunk][kHD + 1];
  __shared__ float rep2[kHD];
  __shared__ float wmax[2];
  __shared__ int widx[2];
  const int c = p.pos != nullptr ? (int)(*p.pos / kChunk) : (int)blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (c >= p.C) return;
  const int64_t vlen = imin64((int64_t)p.lengths[b], p.T);
  const __nv_bfloat16* base = p.k + b * p.skb + h * p.skh;
  const bool vec = (reinterpret_cast<uintptr_t>(base) & 15u) == 0 && p.skn % 8 == 0;
  if (vec) {
    const int piece = tid & 7;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int r = k * 8 + (tid >> 3);
      const int64_t t = (int64_t)c * kChunk + r;
      uint4 w = make_uint4(0u, 0u, 0u, 0u);
      if (t < p.T) w = *reinterpret_cast<const uint4*>(base + t * p.skn + piece * 8);
      const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        xs[r][piece * 8 + 2 * i] = __uint_as_float(u[i] << 16);
        xs[r][piece * 8 + 2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
      }
    }
  } else {
    for (int i = tid; i < kChunk * kHD; i += 64) {
      const int r = i / kHD, d = i % kHD;
      const int64_t t = (int64_t)c * kChunk + r;
      xs[r][d] = t < p.T ? __bfloat162float(base[t * p.skn + d]) : 0.0f;
    }
  }
  __syncthreads();
  // Row energies (row = tid), masked to -inf past the valid length; the first
  // maximum over the rows.
  float e = 0.0f;
#pragma unroll 16
  for (int d = 0; d < kHD; ++d) e = add_rn(e, mul_rn(xs[tid][d], xs[tid][d]));
  e = ((int64_t)c * kChunk + tid < vlen) ? e : -INFINITY;
  float bv = e;
  int bi = tid;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  if (lane == 0) { wmax[warp] = bv; widx[warp] = bi; }
  __syncthreads();
  // Rows 0-31 come before rows 32-63: the second warp wins only when strictly larger.
  const int best_row = wmax[1] > wmax[0] ? widx[1] : widx[0];
  // Masked mean of dim d (= tid) and the blend.
  float s = 0.0f;
  int count = 0;
#pragma unroll 16
  for (int r = 0; r < kChunk; ++r) {
    const bool ok = (int64_t)c * kChunk + r < vlen;
    s = add_rn(s, ok ? xs[r][tid] : 0.0f);
    count += ok;
  }
  const float mean = __fdiv_rn(s, (float)max(count, 1));
  const float rep = add_rn(mul_rn(1.0f - p.alpha, mean), mul_rn(p.alpha, xs[best_row][tid]));
  rep2[tid] = mul_rn(rep, rep);
  __syncthreads();
  float ss = 0.0f;
#pragma unroll 16
  for (int d = 0; d < kHD; ++d) ss = add_rn(ss, rep2[d]);
  const float norm = fmaxf(sqrtf(ss), 1e-6f);
  const bool chunk_valid = (int64_t)c * kChunk < vlen;
  const float v = chunk_valid ? __fdiv_rn(rep, norm) : 0.0f;
  p.reps[((b * p.H + h) * p.C + c) * kHD + tid] = __float2bfloat16_rn(v);
}

// ---------------------------------------------------------------- router

// The tile window of a launch: host-given, or [*pos / 16, + tile_count) read
// from device memory (decode steps replayed from a CUDA graph).
template <typename P>
__device__ __forceinline__ void window_of(const P& p, int64_t& tb, int64_t& te) {
  if (p.pos != nullptr) {
    tb = *p.pos / kTile;
    te = imin64(tb + p.tile_count, p.tiles);
  } else {
    tb = p.tile_begin;
    te = p.tile_end;
  }
}

struct SelectParams {
  const __nv_bfloat16* q; int64_t sqb, sqh, sqn;
  const __nv_bfloat16* reps;  // [B,H,C,64]
  const int32_t* lengths;
  int32_t* top;               // [B,H,tiles,K]
  float* logits;              // optional [B,H,tiles,C], masked (-inf)
  int64_t H, T, C, tiles;
  int64_t tile_begin, tile_end;  // tiles [tile_begin, tile_end) are computed
  int k_slots;
  float temperature;
  const int64_t* pos;            // optional: window [*pos/16, +tile_count) (decode step)
  int64_t tile_count;
};

// Each warp takes one selector tile at a time, kSelRounds tiles in all: the
// CTA's (b, h) representatives are staged in shared memory once for
// kSelRounds * 8 tiles. Arithmetic and summation order are those of the
// reference: the anchor's squares are summed in dimension order (every lane
// runs the same chain), then each lane divides two of its elements.
constexpr int kSelRounds = 4;

__global__ void __launch_bounds__(256) hisa_select_kernel(const SelectParams p) {
  __shared__ float reps[kMaxChunks][kHD + 1];
  __shared__ float anchor[8][kHD];
  const int h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < p.C * kHD; i += blockDim.x)
    reps[i / kHD][i % kHD] = __bfloat162float(p.reps[((b * p.H + h) * p.C) * kHD + i]);
  __syncthreads();
  int64_t tb, te;
  window_of(p, tb, te);
  const int64_t vlen = p.lengths[b];
  for (int r = 0; r < kSelRounds; ++r) {
    const int64_t t = tb + ((int64_t)blockIdx.x * kSelRounds + r) * 8 + warp;
    if (t >= te) break;  // warp-uniform; no block barrier follows
    const int64_t start = t * kTile;
    const int64_t arow = imin64(start, p.T - 1);
    const __nv_bfloat16* qrow = p.q + b * p.sqb + h * p.sqh + arow * p.sqn;
    // F.normalize(anchor.float(), eps=1e-6).to(bf16): float32 sequential norm,
    // IEEE divide, bf16 rounding
    const float x0 = __bfloat162float(qrow[lane]), x1 = __bfloat162float(qrow[lane + 32]);
    __syncwarp();  // the previous round's readers of anchor[warp] are done
    anchor[warp][lane] = mul_rn(x0, x0);
    anchor[warp][lane + 32] = mul_rn(x1, x1);
    __syncwarp();
    float ss = 0.0f;
#pragma unroll
    for (int d = 0; d < kHD; ++d) ss = add_rn(ss, anchor[warp][d]);
    const float nrm = fmaxf(sqrtf(ss), 1e-6f);
    __syncwarp();
    anchor[warp][lane] = round_bf16(__fdiv_rn(x0, nrm));
    anchor[warp][lane + 32] = round_bf16(__fdiv_rn(x1, nrm));
    __syncwarp();
    float val[kMaxChunks / 32];
#pragma unroll
    for (int i = 0; i < kMaxChunks / 32; ++i) {
      const int c = lane + 32 * i;
      float s = -INFINITY;
      if (c < p.C) {
        float acc = 0.0f;
#pragma unroll
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
  const int32_t* top;           // [B,H,tiles,K]
  const __nv_bfloat16* route;   // [B,H,T,4]
  const int32_t* lengths;
  __nv_bfloat16* out; int64_t sob, soh, son;
  int64_t H, T, tiles;
  int64_t tile_begin, tile_end;  // tiles [tile_begin, tile_end) are computed
  int64_t grid_begin;            // tile_begin rounded down to the CTA tile grid
  const int64_t* pos;            // optional: window [*pos/16, +tile_count) (decode step)
  int64_t tile_count;
  int k_slots;
  float* lse;                    // optional [B,H,T]: row log-sum-exp, log2 domain
};

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
    scale[rr] = ex2_approx(m[rr] - msafe[rr]);
    m[rr] = mn;
  }
  float rs[2] = {0.0f, 0.0f};
  uint32_t pa[NT][2];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const float p0 = ex2_approx(s[j][0] - msafe[0]), p1 = ex2_approx(s[j][1] - msafe[0]);
    const float p2 = ex2_approx(s[j][2] - msafe[1]), p3 = ex2_approx(s[j][3] - msafe[1]);
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

// ---------------------------------------------------------------- route prior

struct RouteParams {
  const __nv_bfloat16* q; int64_t sqb, sqh, sqn;
  const __nv_bfloat16* reps;  // [B,H,C,64]
  const int32_t* top;         // [B,H,tiles,K]
  const float* route_scale;   // [H]
  __nv_bfloat16* route;       // [B,H,T,4]
  int64_t H, T, C, tiles;
  int64_t tile_begin, tile_end;  // tiles [tile_begin, tile_end) are computed
  int k_slots;
  const int64_t* pos;            // optional: window [*pos/16, +tile_count) (decode step)
  int64_t tile_count;
};

// One warp per 16-query tile (8 tiles per CTA); two lanes per query row, lane
// 2i + hf holding dims [32 hf, 32 hf + 32) of row i. Every float32 sum keeps the
// reference's order over the 64 dims: the even lane sums dims 0-31 and hands its
// partial to the odd lane (one shuffle), which continues with dims 32-63.
__global__ void __launch_bounds__(256) hisa_route_kernel(const RouteParams p) {
  __shared__ float rsel[8][kTopK][kHD];
  __shared__ int sel[8][kTopK];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hf = lane & 1, ri = lane >> 1;
  const int h = blockIdx.y, b = blockIdx.z;
  int64_t tb, te;
  window_of(p, tb, te);
  const int64_t t = tb + (int64_t)blockIdx.x * 8 + warp;
  const bool tile_ok = t < te;
  const int64_t row = t * kTile + ri;
  // Issue the half-row load first; the selections and representatives follow.
  uint4 qw[4];
  {
    const int64_t r = row < p.T ? row : p.T - 1;
    const uint4* src = reinterpret_cast<const uint4*>(p.q + b * p.sqb + h * p.sqh + r * p.sqn + 32 * hf);
#pragma unroll
    for (int i = 0; i < 4; ++i) qw[i] = src[i];
  }
  if (lane < kTopK) sel[warp][lane] = (tile_ok && lane < p.k_slots) ? p.top[((b * p.H + h) * p.tiles + t) * p.k_slots + lane] : -1;
  __syncwarp();
  for (int x = lane; x < kTopK * kHD; x += 32) {
    const int k = x / kHD, c = sel[warp][k];
    rsel[warp][k][x % kHD] = c >= 0 ? __bfloat162float(p.reps[((b * p.H + h) * p.C + c) * kHD + x % kHD]) : 0.0f;
  }
  __syncwarp();
  if (!tile_ok) return;  // warp-uniform
  const bool row_ok = row < p.T;
  float qh[32];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t u[4] = {qw[i].x, qw[i].y, qw[i].z, qw[i].w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      qh[8 * i + 2 * k] = __uint_as_float(u[k] << 16);
      qh[8 * i + 2 * k + 1] = __uint_as_float(u[k] & 0xffff0000u);
    }
  }
  const unsigned pair = 0xffffffffu;
  const int even = lane & ~1;
  // q^ = bf16(q / max(|q|, 1e-6)): sequential float32 norm, IEEE divide.
  float ss = 0.0f;
  if (hf == 0) {
#pragma unroll
    for (int d = 0; d < 32; ++d) ss = add_rn(ss, mul_rn(qh[d], qh[d]));
  }
  ss = __shfl_sync(pair, ss, even);
  if (hf == 1) {
#pragma unroll
    for (int d = 0; d < 32; ++d) ss = add_rn(ss, mul_rn(qh[d], qh[d]));
  }
  ss = __shfl_sync(pair, ss, even | 1);
  const float nrm = fmaxf(sqrtf(ss), 1e-6f);
#pragma unroll
  for (int d = 0; d < 32; ++d) qh[d] = round_bf16(__fdiv_rn(qh[d], nrm));
  float sc[kTopK];
#pragma unroll
  for (int k = 0; k < kTopK; ++k) {
    const float* r = rsel[warp][k] + 32 * hf;
    float acc = 0.0f;
    if (hf == 0) {
#pragma unroll
      for (int d = 0; d < 32; ++d) acc = add_rn(acc, mul_rn(qh[d], r[d]));
    }
    acc = __shfl_sync(pair, acc, even);
    if (hf == 1) {
#pragma unroll
      for (int d = 0; d < 32; ++d) acc = add_rn(acc, mul_rn(qh[d], r[d]));
    }
    sc[k] = acc;  // complete in the odd lane
  }
  if (hf == 0 || !row_ok) return;
  float sum = 0.0f;
  int count = 0;
#pragma unroll
  for (int k = 0; k < kTopK; ++k) {
    const bool ok = sel[warp][k] >= 0;
    sum = add_rn(sum, ok ? sc[k] : 0.0f);
    count += ok;
  }
  const float mean = __fdiv_rn(sum, (float)max(count, 1));
  const float scale = p.route_scale[h];
  uint32_t packed[2];
#pragma unroll
  for (int k = 0; k < kTopK; k += 2) {
    const float v0 = sel[warp][k] >= 0 ? mul_rn(__fsub_rn(sc[k], mean), scale) : 0.0f;
    const float v1 = sel[warp][k + 1] >= 0 ? mul_rn(__fsub_rn(sc[k + 1], mean), scale) : 0.0f;
    const __nv_bfloat162 two = __floats2bfloat162_rn(v0, v1);
    packed[k / 2] = *reinterpret_cast<const uint32_t*>(&two);
  }
  *reinterpret_cast<uint2*>(p.route + ((b * p.H + h) * p.T + row) * kTopK) = make_uint2(packed[0], packed[1]);
}

// ---------------------------------------------------------------- pipelined tile attention
//
// CTA = 8 selector tiles (128 queries) of one (b, h): warps 0-7 each own one
// 16-query tile; lane 0 of warp 0 also issues the chunk loads. The CTA's key chunks -- the three
// 64-row blocks of local keys around its queries and the union of the
// routed chunks its tiles selected -- are listed once, fetched once by TMA
// (K and V boxes of 64 rows x 64 dims, 128-byte swizzle) into a ring of
// kStages stages, and consumed by every tile that needs them (mma.sync,
// online softmax), so loads of later chunks overlap the math of earlier ones
// and neighbouring tiles share their local and routed chunks.

constexpr int kCtaTiles = 8;
constexpr int kStages = 5;
constexpr int kStageBytes = 2 * 64 * 128;  // K and V boxes
constexpr int kMaxEntries = 3 + kCtaTiles * kTopK;
constexpr uint32_t kWait = 1u << 24;

struct ChunkEntry {
  int32_t row0;   // first key row
  int8_t global;  // 0: local K/V, 1: global (adapted) K/V
  uint8_t mask;   // tiles that attend to this chunk
  int8_t slot[kCtaTiles];  // routed: the tile's top-k slot (route prior), else -1
};

struct AttnSmem {
  static constexpr uint32_t ring = 0;
  static constexpr uint32_t route = kStages * kStageBytes;  // [8 tiles][16][4] fp32
  static constexpr uint32_t entries = route + kCtaTiles * 16 * kTopK * 4;
  static constexpr uint32_t bars = entries + kMaxEntries * sizeof(ChunkEntry);
  static constexpr uint32_t count = bars + 2 * kStages * 8;
  static constexpr uint32_t bytes = count + 8 + 4 * kCtaTiles * kTopK + 1024;  // + alignment slack
};

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(n) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile("{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}"
               : "=r"(done) : "r"(bar), "r"(parity) : "memory");
  return done != 0;
}
// Bounded wait; raises the CTA's abort flag after kWait polls or when another warp has.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  for (uint32_t it = 0; it < kWait; ++it) {
    if (mbar_try(bar, parity)) return true;
    if (*abort_flag) return false;
  }
  *abort_flag = 1;
  return false;
}
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, int w,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(bar) : "memory");
}

struct AttnMaps {
  CUtensorMap lk, lv, gk, gv;
};

__global__ void __launch_bounds__(kCtaTiles * 32, 2)
hisa_attn_kernel(const AttnParams p, const __grid_constant__ AttnMaps maps, int32_t* status) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* smem = smem_raw + (base - raw);
  float* s_route = reinterpret_cast<float*>(smem + AttnSmem::route);
  ChunkEntry* s_ent = reinterpret_cast<ChunkEntry*>(smem + AttnSmem::entries);
  const uint32_t bar_full = base + AttnSmem::bars, bar_empty = bar_full + 8 * kStages;
  int* s_count = reinterpret_cast<int*>(smem + AttnSmem::count);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + AttnSmem::count + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, b = blockIdx.z;
  // CTAs cover aligned groups of kCtaTiles tiles whatever the window, so a
  // windowed launch visits each tile's chunks in the order a full launch does
  // (bit-identical rows); tiles of a group outside the window stay idle.
  int64_t tb, te;
  window_of(p, tb, te);
  const int64_t gb = p.pos != nullptr ? tb - tb % kCtaTiles : p.grid_begin;
  const int64_t T0 = (gb + (int64_t)blockIdx.x * kCtaTiles) * kTile;
  if (T0 / kTile >= te) return;  // whole CTA, before any barrier (device windows size the grid up)
  auto in_window = [&](int64_t t) { return t >= tb && t < te; };
  const int64_t vlen = imin64((int64_t)p.lengths[b], p.T);
  const int32_t* top = p.top + ((int64_t)b * p.H + h) * p.tiles * p.k_slots;

  // ---- phase A: the CTA's 32 (tile, slot) selections into smem
  int* s_top = s_count + 2;  // [kCtaTiles * kTopK]
  if (warp == 0) {
    const int i = lane / kTopK, k = lane % kTopK;
    const int64_t t = T0 / kTile + i;
    s_top[lane] = (in_window(t) && k < p.k_slots) ? top[t * p.k_slots + k] : -1;
  }
  __syncthreads();
  // ---- phase B: chunk list + barriers (warp 0), route prior rows (everyone)
  if (warp == 0) {
    // Local chunks: the three 64-row blocks of [T0 - 64, T0 + 128).
    int n = 0;
    if (lane == 0) {
      for (int k = 0; k < 3; ++k) {
        const int64_t row0 = T0 - 64 + 64 * k;
        if (row0 >= p.T || row0 + 64 <= 0) continue;
        ChunkEntry e;
        e.row0 = (int32_t)row0;
        e.global = 0;
        e.mask = 0;
        for (int i = 0; i < kCtaTiles; ++i) {
          e.slot[i] = -1;
          const int64_t t0 = T0 + kTile * i;
          if (t0 < p.T && in_window(t0 / kTile) && t0 - 64 < row0 + 64 && row0 < t0 + kTile)
            e.mask |= (uint8_t)(1u << i);
        }
        if (e.mask) s_ent[n++] = e;
      }
    }
    n = __shfl_sync(0xffffffffu, n, 0);
    // Routed chunks: one entry per distinct chunk id among the 32 selections
    // (lane = tile * 4 + slot); the lowest lane of each group of equal ids
    // writes the entry, in ascending chunk order -- so each tile meets its own
    // chunks in the same order whichever tiles share the CTA (a windowed
    // launch reproduces a full launch bit for bit).
    const int c = s_top[lane];
    const unsigned same = __match_any_sync(0xffffffffu, c);
    const bool leader = c >= 0 && (__ffs(same) - 1) == lane;
    const unsigned leaders = __ballot_sync(0xffffffffu, leader);
    int rank = 0;
    for (int j = 0; j < 32; ++j) {
      const int cj = __shfl_sync(0xffffffffu, c, j);
      rank += ((leaders >> j) & 1u) && cj < c;
    }
    if (leader) {
      ChunkEntry e;
      e.row0 = c * kChunk;
      e.global = 1;
      e.mask = 0;
      for (int k = 0; k < kCtaTiles; ++k) e.slot[k] = -1;
      for (unsigned m = same; m; m &= m - 1) {
        const int ln = __ffs(m) - 1;
        e.mask |= (uint8_t)(1u << (ln / kTopK));
        e.slot[ln / kTopK] = (int8_t)(ln % kTopK);
      }
      s_ent[n + rank] = e;
    }
    if (lane == 0) {
      *s_count = n + __popc(leaders);
      *abort_flag = 0;
      for (int s = 0; s < kStages; ++s) {
        mbar_init(bar_full + 8 * s, 1);
        mbar_init(bar_empty + 8 * s, kCtaTiles);
      }
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
  }
  // Route prior of the CTA's 128 query rows (4 slots each).
  for (int x = threadIdx.x; x < kCtaTiles * 16 * kTopK; x += blockDim.x) {
    const int64_t row = T0 + x / kTopK;
    s_route[x] = row < p.T ? __bfloat162float(p.route[(((int64_t)b * p.H + h) * p.T + row) * kTopK + x % kTopK]) : 0.0f;
  }
  __syncthreads();
  const int n_ent = *s_count;

  // Chunk e goes to stage e % kStages; its loads are issued once every tile
  // has released the chunk that used the stage before it.
  auto issue = [&](int e) {
    const int s = e % kStages;
    const uint32_t dst = base + AttnSmem::ring + s * kStageBytes;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar_full + 8 * s),
                 "r"(kStageBytes) : "memory");
    const ChunkEntry& en = s_ent[e];
    tma_load_4d(dst, en.global ? &maps.gk : &maps.lk, 0, en.row0, h, b, bar_full + 8 * s);
    tma_load_4d(dst + kStageBytes / 2, en.global ? &maps.gv : &maps.lv, 0, en.row0, h, b, bar_full + 8 * s);
  };
  int issued = 0;  // thread 0: entries whose loads were issued
  if (threadIdx.x == 0)
    for (int e = 0; e < n_ent && e < kStages; ++e) { issue(e); issued = e + 1; }
  {
    // ---------------- one 16-query tile per warp
    const int tile = warp;
    const int64_t t0 = T0 + (int64_t)kTile * tile;
    const int g = lane >> 2, t4 = lane & 3;
    const __nv_bfloat16* qb = p.q + b * p.sqb + h * p.sqh;
    const bool tile_ok = t0 < p.T && in_window(t0 / kTile);
    float* route = s_route + tile * 16 * kTopK;
    // Q fragments (m16n8k16 A operand) straight from global.
    uint32_t qa[4][4];
    {
      const int64_t ra = imin64(t0 + g, p.T - 1), rb = imin64(t0 + g + 8, p.T - 1);
#pragma unroll
      for (int kt = 0; kt < 4; ++kt) {
        const int c0 = kt * 16 + 2 * t4;
        qa[kt][0] = *reinterpret_cast<const uint32_t*>(qb + ra * p.sqn + c0);
        qa[kt][1] = *reinterpret_cast<const uint32_t*>(qb + rb * p.sqn + c0);
        qa[kt][2] = *reinterpret_cast<const uint32_t*>(qb + ra * p.sqn + c0 + 8);
        qa[kt][3] = *reinterpret_cast<const uint32_t*>(qb + rb * p.sqn + c0 + 8);
      }
    }
    float o[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};

    for (int e = 0; e < n_ent; ++e) {
      const int s = e % kStages;
      const uint32_t ph = (uint32_t)(e / kStages) & 1u;
      // One lane waits; the outcome is the warp's, so the warp leaves together.
      const bool ready = __shfl_sync(0xffffffffu, lane == 0 ? (int)mbar_wait(bar_full + 8 * s, ph, abort_flag) : 0, 0);
      if (!ready) break;
      const ChunkEntry& en = s_ent[e];
      if (tile_ok && ((en.mask >> tile) & 1)) {
        const uint32_t ktile = base + AttnSmem::ring + s * kStageBytes;
        const uint32_t vtile = ktile + kStageBytes / 2;
        const int row0i = en.row0, t0i = (int)t0, vleni = (int)vlen;
        if (en.global) {
          const int slot = en.slot[tile];
          const float bias[2] = {route[g * kTopK + slot], route[(g + 8) * kTopK + slot]};
          auto mask = [&](int r, int i) {
            const int id = row0i + i, n = t0i + r;
            return id < n - kWindow && id < vleni && n < vleni;
          };
          attend_block<8>(qa, ktile, vtile, bias, mask, o, m, l, lane);
        } else {
          const float bias[2] = {0.0f, 0.0f};
          auto mask = [&](int r, int i) {
            const int id = row0i + i, n = t0i + r;
            return id >= n - kWindow && id < n && id >= 0 && id < vleni && n < vleni;
          };
          attend_block<8>(qa, ktile, vtile, bias, mask, o, m, l, lane);
        }
      }
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar_empty + 8 * s) : "memory");
      if (threadIdx.x == 0 && e + kStages < n_ent && mbar_wait(bar_empty + 8 * s, ph, abort_flag)) {
        issue(e + kStages);
        issued = e + kStages + 1;
      }
    }
    // Leave no copy in flight: of the issued entries, all but the last kStages
    // were released by every tile (so they landed); wait for those kStages,
    // whether the loop finished or an abort ended it early.
    if (threadIdx.x == 0)
      for (int e = issued > kStages ? issued - kStages : 0; e < issued; ++e)
        for (uint32_t it = 0; it < kWait && !mbar_try(bar_full + 8 * (e % kStages), (uint32_t)(e / kStages) & 1u); ++it) {}

    // Epilogue: O / l in bf16; rows past the valid length are zero.
    if (tile_ok) {
      __nv_bfloat16* ob = p.out + b * p.sob + h * p.soh;
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const int64_t row = t0 + g + rr * 8;
        if (row >= p.T) continue;
        const float inv = (l[rr] > 0.0f && row < vlen) ? 1.0f / l[rr] : 0.0f;
        if (p.lse != nullptr && t4 == 0)
          p.lse[((int64_t)b * p.H + h) * p.T + row] = (l[rr] > 0.0f && row < vlen) ? m[rr] + __log2f(l[rr]) : INFINITY;
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          const uint32_t v = pack_bf16(o[n][rr * 2] * inv, o[n][rr * 2 + 1] * inv);
          *reinterpret_cast<uint32_t*>(ob + row * p.son + n * 8 + 2 * t4) = v;
        }
      }
    }
  }
  if (*abort_flag && lane == 0 && status != nullptr) atomicExch(status, DWARF_DEVICE_TIMEOUT);
}

// ---------------------------------------------------------------- tcgen05 tile attention
//
// The same CTA (8 selector tiles = 128 queries of one (b, h)) and chunk list
// as hisa_attn_kernel, with the dense tile products on the 5th-generation
// tensor cores and their accumulators in tensor memory:
//   warp 0      chunk list (once), then TMA producer: the Q tile (128 rows)
//               once, and each chunk's K and V boxes (64 rows x 64 dims,
//               128-byte swizzle) into a kTcStages ring;
//   warp 1      allocates 256 TMEM columns and issues, from one thread,
//                 S_e = Q . K_e^T   (M = 128 queries, N = 64 keys, K = 64)
//                 into S[e % 2] (columns 0 / 64), and, once the softmax has
//                 written P_e, O_e = P_e . V_e (M = 128, N = 64 dims,
//                 K = 64 keys; V read in place as an MN-major operand) into
//                 O[e % 2] (columns 128 / 192);
//   warps 2-5   one query row per thread (TMEM lane = row): read S_e with
//               tcgen05.ld, apply the lane masks, the route prior and the
//               scale, run the online-softmax update, write P_e (bf16) to a
//               swizzled shared-memory tile, and fold O_e into the fp32 row
//               accumulator in registers (O = alpha_e * O + O_e) one chunk
//               behind, so S_{e+1} and O_e overlap the softmax of chunk e.
// A warp skips the chunks none of its 32 rows attend, and a row folds only
// the chunks it attended: a tile meets its own chunks in list order whichever
// tiles share the CTA, as in hisa_attn_kernel (windowed launches reproduce
// full ones bit for bit).
// Every wait is bounded; a timeout aborts all roles, drains the copies and
// MMAs in flight, frees tensor memory and records DWARF_DEVICE_TIMEOUT.
constexpr int kTcStages = 3;
constexpr int kTcThreads = 192;
constexpr uint32_t kTcCols = 256;

struct TcSmem {
  static constexpr uint32_t q = 0;                                 // 128 rows x 128 B
  static constexpr uint32_t ring = q + 128 * 128;                  // stages: K box, V box
  static constexpr uint32_t pbuf = ring + kTcStages * kStageBytes;  // P[2]: 128 rows x 128 B
  static constexpr uint32_t route = pbuf + 2 * 128 * 128;          // [128 rows][4] fp32
  static constexpr uint32_t entries = route + 128 * kTopK * 4;
  static constexpr uint32_t bars = (entries + kMaxEntries * sizeof(ChunkEntry) + 7) / 8 * 8;
  // q, full[S], empty[S], s_full[2], p_full[2], o_full[2], o_empty[2], drain
  static constexpr uint32_t misc = bars + (2 + 2 * kTcStages + 8) * 8;
  static constexpr uint32_t bytes = misc + 16 + 4 * 32 + 1024;  // + alignment slack
};

__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr) {
  // 128-byte swizzle, 8-row (1024-byte) atoms; for the K-major operands the
  // stride field steps between 8-row groups of M/N, for the MN-major V between
  // 8-row groups of K (keys). The leading field is unused (one atom along
  // K for K-major, one 64-element atom along N for MN-major).
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
// kind::f16 instruction descriptor: bf16 A and B, fp32 D, M x N; b_mn: B is MN-major.
__host__ __device__ constexpr uint32_t tc_idesc(int M, int N, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (b_mn ? (1u << 16) : 0u) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ void tc_mma1(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile("{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\ntcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
               ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(acc) : "memory");
}
__device__ __forceinline__ void tc_commit1(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive1(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// 32 consecutive fp32 columns of this thread's TMEM lane (load and wait in one statement).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr) : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// (d0, d1) = (a0, a1) * (b0, b1) + (c0, c1) as one packed fp32x2 FMA.
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0,
                                      float c1) {
  asm("{\n.reg .b64 pa, pb, pc;\nmov.b64 pa, {%2, %3};\nmov.b64 pb, {%4, %5};\nmov.b64 pc, {%6, %7};\n"
      "fma.rn.f32x2 pc, pa, pb, pc;\nmov.b64 {%0, %1}, pc;\n}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}

struct TcMaps {
  CUtensorMap q, lk, lv, gk, gv;
};

__global__ void __launch_bounds__(kTcThreads, 2)
hisa_attn_tc_kernel(const AttnParams p, const __grid_constant__ TcMaps maps, int32_t* status) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* smem = smem_raw + (base - raw);
  float* s_route = reinterpret_cast<float*>(smem + TcSmem::route);
  ChunkEntry* s_ent = reinterpret_cast<ChunkEntry*>(smem + TcSmem::entries);
  const uint32_t bar_q = base + TcSmem::bars;
  const uint32_t bar_full = bar_q + 8, bar_empty = bar_full + 8 * kTcStages;
  const uint32_t bar_sfull = bar_empty + 8 * kTcStages, bar_pfull = bar_sfull + 16;
  const uint32_t bar_ofull = bar_pfull + 16, bar_oempty = bar_ofull + 16, bar_drain = bar_oempty + 16;
  int* s_count = reinterpret_cast<int*>(smem + TcSmem::misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + TcSmem::misc + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + TcSmem::misc + 8);
  int* s_top = reinterpret_cast<int*>(smem + TcSmem::misc + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, b = blockIdx.z;
  int64_t tb, te;
  window_of(p, tb, te);
  const int64_t gb = p.pos != nullptr ? tb - tb % kCtaTiles : p.grid_begin;
  const int64_t T0 = (gb + (int64_t)blockIdx.x * kCtaTiles) * kTile;
  if (T0 / kTile >= te) return;  // whole CTA, before any barrier or allocation
  auto in_window = [&](int64_t t) { return t >= tb && t < te; };
  const int64_t vlen = imin64((int64_t)p.lengths[b], p.T);
  const int32_t* top = p.top + ((int64_t)b * p.H + h) * p.tiles * p.k_slots;

  // ---- the CTA's 32 (tile, slot) selections, then its chunk list (as hisa_attn_kernel)
  if (warp == 0) {
    const int i = lane / kTopK, k = lane % kTopK;
    const int64_t t = T0 / kTile + i;
    s_top[lane] = (in_window(t) && k < p.k_slots) ? top[t * p.k_slots + k] : -1;
  }
  __syncthreads();
  if (warp == 0) {
    int n = 0;
    if (lane == 0) {
      for (int k = 0; k < 3; ++k) {
        const int64_t row0 = T0 - 64 + 64 * k;
        if (row0 >= p.T || row0 + 64 <= 0) continue;
        ChunkEntry e;
        e.row0 = (int32_t)row0;
        e.global = 0;
        e.mask = 0;
        for (int i = 0; i < kCtaTiles; ++i) {
          e.slot[i] = -1;
          const int64_t t0 = T0 + kTile * i;
          if (t0 < p.T && in_window(t0 / kTile) && t0 - 64 < row0 + 64 && row0 < t0 + kTile)
            e.mask |= (uint8_t)(1u << i);
        }
        if (e.mask) s_ent[n++] = e;
      }
    }
    n = __shfl_sync(0xffffffffu, n, 0);
    const int c = s_top[lane];
    const unsigned same = __match_any_sync(0xffffffffu, c);
    const bool leader = c >= 0 && (__ffs(same) - 1) == lane;
    const unsigned leaders = __ballot_sync(0xffffffffu, leader);
    int rank = 0;
    for (int j = 0; j < 32; ++j) {
      const int cj = __shfl_sync(0xffffffffu, c, j);
      rank += ((leaders >> j) & 1u) && cj < c;
    }
    if (leader) {
      ChunkEntry e;
      e.row0 = c * kChunk;
      e.global = 1;
      e.mask = 0;
      for (int k = 0; k < kCtaTiles; ++k) e.slot[k] = -1;
      for (unsigned m = same; m; m &= m - 1) {
        const int ln = __ffs(m) - 1;
        e.mask |= (uint8_t)(1u << (ln / kTopK));
        e.slot[ln / kTopK] = (int8_t)(ln % kTopK);
      }
      s_ent[n + rank] = e;
    }
    if (lane == 0) {
      *s_count = n + __popc(leaders);
      *abort_flag = 0;
      mbar_init(bar_q, 1);
      for (int s = 0; s < kTcStages; ++s) {
        mbar_init(bar_full + 8 * s, 1);
        mbar_init(bar_empty + 8 * s, 1);
      }
      for (int i = 0; i < 2; ++i) {
        mbar_init(bar_sfull + 8 * i, 1);
        mbar_init(bar_pfull + 8 * i, 128);
        mbar_init(bar_ofull + 8 * i, 1);
        mbar_init(bar_oempty + 8 * i, 128);
      }
      mbar_init(bar_drain, 1);
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
  } else if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTcCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  for (int x = threadIdx.x; x < kCtaTiles * 16 * kTopK; x += blockDim.x) {
    const int64_t row = T0 + x / kTopK;
    s_route[x] = row < p.T ? __bfloat162float(p.route[(((int64_t)b * p.H + h) * p.T + row) * kTopK + x % kTopK]) : 0.0f;
  }
  tc_before();
  __syncthreads();
  tc_after();
  const int n_ent = *s_count;
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar_q), "r"(128 * 128) : "memory");
      tma_load_4d(base + TcSmem::q, &maps.q, 0, (int)T0, h, b, bar_q);
      tma_load_4d(base + TcSmem::q + 64 * 128, &maps.q, 0, (int)T0 + 64, h, b, bar_q);
      int issued = 0;
      for (int e = 0; e < n_ent; ++e) {
        const int s = e % kTcStages;
        if (!mbar_wait(bar_empty + 8 * s, ((uint32_t)(e / kTcStages) & 1u) ^ 1u, abort_flag)) break;
        const uint32_t dst = base + TcSmem::ring + s * kStageBytes;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar_full + 8 * s),
                     "r"(kStageBytes) : "memory");
        const ChunkEntry& en = s_ent[e];
        tma_load_4d(dst, en.global ? &maps.gk : &maps.lk, 0, en.row0, h, b, bar_full + 8 * s);
        tma_load_4d(dst + kStageBytes / 2, en.global ? &maps.gv : &maps.lv, 0, en.row0, h, b, bar_full + 8 * s);
        issued = e + 1;
      }
      // Leave no copy in flight: the Q tile and the last kTcStages issued chunks
      // (every earlier one was consumed, hence landed) have arrived.
      for (uint32_t it = 0; it < kWait && !mbar_try(bar_q, 0); ++it) {}
      for (int e = issued > kTcStages ? issued - kTcStages : 0; e < issued; ++e)
        for (uint32_t it = 0; it < kWait && !mbar_try(bar_full + 8 * (e % kTcStages), (uint32_t)(e / kTcStages) & 1u);
             ++it) {}
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdS = tc_idesc(128, 64, false), kIdO = tc_idesc(128, 64, true);
      const uint32_t q_s = base + TcSmem::q;
      bool ok = mbar_wait(bar_q, 0, abort_flag);
      auto issue_s = [&](int e) -> bool {
        const int s = e % kTcStages;
        if (!mbar_wait(bar_full + 8 * s, (uint32_t)(e / kTcStages) & 1u, abort_flag)) return false;
        tc_after();
        const uint32_t k_s = base + TcSmem::ring + s * kStageBytes;
        const uint32_t d = tmem + (uint32_t)(e & 1) * 64u;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) tc_mma1(d, tc_desc(q_s + kk * 32), tc_desc(k_s + kk * 32), kIdS, kk != 0);
        tc_commit1(bar_sfull + 8 * (e & 1));
        return true;
      };
      if (ok) tc_after();
      for (int e = 0; ok && e < n_ent && e < 2; ++e) ok = issue_s(e);
      for (int e = 0; ok && e < n_ent; ++e) {
        const int buf = e & 1;
        const uint32_t ph = (uint32_t)(e >> 1) & 1u;
        if (!(ok = mbar_wait(bar_pfull + 8 * buf, ph, abort_flag))) break;
        if (!(ok = mbar_wait(bar_oempty + 8 * buf, ph ^ 1u, abort_flag))) break;
        tc_after();
        const int s = e % kTcStages;
        const uint32_t v_s = base + TcSmem::ring + s * kStageBytes + kStageBytes / 2;
        const uint32_t p_s = base + TcSmem::pbuf + buf * 128 * 128;
        const uint32_t d = tmem + 128u + (uint32_t)buf * 64u;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) tc_mma1(d, tc_desc(p_s + kk * 32), tc_desc(v_s + kk * 2048), kIdO, kk != 0);
        tc_commit1(bar_ofull + 8 * buf);
        tc_commit1(bar_empty + 8 * s);
        if (e + 2 < n_ent) ok = issue_s(e + 2);  // S[e % 2] was read before P_e was published
      }
      // Drain: every MMA issued so far has completed once this commit lands.
      tc_commit1(bar_drain);
      for (uint32_t it = 0; it < kWait && !mbar_try(bar_drain, 0); ++it) {}
    }
    __syncwarp();
  } else {
    // ---------------- softmax / accumulation: one query row per thread
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int tile = row >> 4;
    const int64_t n = T0 + row;
    const bool tile_ok = T0 + kTile * tile < p.T && in_window((T0 + kTile * tile) / kTile);
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    const int ni = (int)n, vleni = (int)vlen;
    float o[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) o[i] = 0.0f;
    float m = -INFINITY, l = 0.0f, alpha_prev = 1.0f;
    bool act_prev = false, ok = true;
    constexpr float kC1 = 0.125f * kLog2e;
    // Waits and tensor-memory loads are warp-wide (tcgen05.ld is .sync.aligned):
    // every lane polls, and the warp goes on only if all of them saw the phase.
    auto warp_wait = [&](uint32_t bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
    };
    // O = alpha_e * O + O_e for rows that attended chunk e, then free O[e % 2].
    auto fold = [&](int e) -> bool {
      const int buf = e & 1;
      if (!warp_wait(bar_ofull + 8 * buf, (uint32_t)(e >> 1) & 1u)) return false;
      tc_after();
      if (__any_sync(0xffffffffu, act_prev)) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          float v[32];
          tmem_ld32(lane_addr + 128u + (uint32_t)buf * 64u + half * 32, v);
          if (act_prev) {
#pragma unroll
            for (int i = 0; i < 32; i += 2)
              ffma2(o[half * 32 + i], o[half * 32 + i + 1], alpha_prev, alpha_prev, o[half * 32 + i],
                    o[half * 32 + i + 1], v[i], v[i + 1]);
          }
        }
      }
      tc_before();
      mbar_arrive1(bar_oempty + 8 * buf);
      return true;
    };
    for (int e = 0; e < n_ent; ++e) {
      const int buf = e & 1;
      if (!(ok = warp_wait(bar_sfull + 8 * buf, (uint32_t)(e >> 1) & 1u))) break;
      tc_after();
      const ChunkEntry& en = s_ent[e];
      int lo, hi;  // valid keys of this row: index i of the chunk in [lo, hi)
      float bias = 0.0f;
      if (en.global) {
        lo = 0;
        hi = min(ni - kWindow, vleni) - en.row0;
        bias = s_route[row * kTopK + (en.slot[tile] >= 0 ? en.slot[tile] : 0)];
      } else {
        lo = max(ni - kWindow, 0) - en.row0;
        hi = min(ni, vleni) - en.row0;
      }
      const bool want = tile_ok && ((en.mask >> tile) & 1) && ni < vleni && hi > lo && hi > 0 && lo < 64;
      float alpha = 1.0f;
      if (__any_sync(0xffffffffu, want)) {  // warp-uniform: the whole warp loads its 32 rows
        float sv[64];
        tmem_ld32(lane_addr + (uint32_t)buf * 64u, *reinterpret_cast<float(*)[32]>(sv));
        tmem_ld32(lane_addr + (uint32_t)buf * 64u + 32, *reinterpret_cast<float(*)[32]>(sv + 32));
        if (want) {
          const float c2 = bias * kLog2e;
#pragma unroll
          for (int i = 0; i < 64; i += 2) ffma2(sv[i], sv[i + 1], sv[i], sv[i + 1], kC1, kC1, c2, c2);
          if (lo > 0 || hi < 64) {
#pragma unroll
            for (int i = 0; i < 64; ++i)
              if ((unsigned)(i - lo) >= (unsigned)(hi - lo)) sv[i] = -INFINITY;
          }
          float mx = sv[0];
#pragma unroll
          for (int i = 1; i < 64; ++i) mx = fmaxf(mx, sv[i]);
          const float mn = fmaxf(m, mx);
          alpha = ex2_approx(m - mn);  // m = -inf on the row's first chunk: 0
          m = mn;
          float rs0 = 0.0f, rs1 = 0.0f;
          // P row (bf16) -> swizzled tile: 16-byte chunk c of row r at chunk c ^ (r & 7)
          unsigned char* prow = smem + TcSmem::pbuf + buf * 128 * 128 + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint32_t w[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float p0 = ex2_approx(sv[8 * c + 2 * k] - mn), p1 = ex2_approx(sv[8 * c + 2 * k + 1] - mn);
              rs0 += p0;
              rs1 += p1;
              w[k] = pack_bf16(p0, p1);
            }
            *reinterpret_cast<uint4*>(prow + ((c ^ (row & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
          }
          l = l * alpha + (rs0 + rs1);
        }
      }
      // Rows that skip chunk e leave their (stale) P row: fold() does not read their O_e.
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_before();
      mbar_arrive1(bar_pfull + 8 * buf);
      if (e >= 1 && !(ok = fold(e - 1))) break;
      alpha_prev = alpha;
      act_prev = want;
    }
    if (ok && n_ent > 0) ok = fold(n_ent - 1);
    if (ok && !*abort_flag && tile_ok && n < p.T) {
      const float inv = (l > 0.0f && n < vlen) ? 1.0f / l : 0.0f;
      __nv_bfloat16* orow = p.out + (int64_t)b * p.sob + (int64_t)h * p.soh + n * p.son;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 w;
        w.x = pack_bf16(o[8 * c] * inv, o[8 * c + 1] * inv);
        w.y = pack_bf16(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
        w.z = pack_bf16(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
        w.w = pack_bf16(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
        *reinterpret_cast<uint4*>(orow + 8 * c) = w;
      }
      if (p.lse != nullptr)
        p.lse[((int64_t)b * p.H + h) * p.T + n] = (l > 0.0f && n < vlen) ? m + __log2f(l) : INFINITY;
    }
  }
  tc_before();
  __syncthreads();
  if (warp == 1) {
    tc_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcCols) : "memory");
  }
  if (*abort_flag && threadIdx.x == 0 && status != nullptr) atomicExch(status, DWARF_DEVICE_TIMEOUT);
}

// 4-D bf16 tensor map over a [B, H, T, 64] view (element strides sb, sh, sn),
// box 64 rows x 64 dims, 128-byte swizzle.
bool make_kv_map(CUtensorMap* map, const void* ptr, int64_t B, int64_t H, int64_t T, int64_t sb, int64_t sh,
                 int64_t sn) {
  auto fn = tensormap_encoder();
  if (fn == nullptr) return false;
  const cuuint64_t dims[4] = {64, (cuuint64_t)T, (cuuint64_t)H, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)sn * 2, (cuuint64_t)sh * 2, (cuuint64_t)sb * 2};
  const cuuint32_t box[4] = {64, 64, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool al16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

// Tile window [begin, begin + count) of `tiles` (count 0: to the end).
bool tile_window(int64_t begin, int64_t count, int64_t tiles, int64_t* b, int64_t* e) {
  if (begin < 0 || count < 0 || begin > tiles) return false;
  const int64_t end = count == 0 ? tiles : begin + count;
  if (end > tiles) return false;
  *b = begin;
  *e = end;
  return true;
}

// Host side of a launch's tile window: [begin, begin + count) checked against
// the tile count, or with a device position the count alone (>= 1; the
// kernel clips the window at the last tile).
template <typename P>
bool launch_window(int64_t begin, int64_t count, const int64_t* pos, P* p, int64_t* n_tiles) {
  p->pos = pos;
  p->tile_count = count;
  if (pos != nullptr) {
    if (count < 1 || count > p->tiles) return false;
    p->tile_begin = 0;
    p->tile_end = count;
    *n_tiles = count;
    return true;
  }
  if (!tile_window(begin, count, p->tiles, &p->tile_begin, &p->tile_end)) return false;
  *n_tiles = p->tile_end - p->tile_begin;
  return true;
}

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
               a->H, a->T, (a->T + kChunk - 1) / kChunk, a->blend_alpha, a->pos};
  dim3 grid(a->pos != nullptr ? 1u : (unsigned)p.C, (unsigned)a->H, (unsigned)a->B);
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
  int64_t n_tiles = 0;
  if (!launch_window(a->tile_begin, a->tile_count, a->pos, &p, &n_tiles)) return DWARF_ERR_SHAPE;
  if (n_tiles == 0) return DWARF_OK;
  const int64_t per_cta = 8 * kSelRounds;
  dim3 grid((unsigned)((n_tiles + per_cta - 1) / per_cta), (unsigned)a->H, (unsigned)a->B);
  hisa_select_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(p);
  return launch_status();
}

extern "C" int dwarf_hisa_route(const dwarf_hisa_route_args* a, void* stream) {
  DWARF_CHECK_VERSION(a);
  if (a->head_dim != kHD || a->selector_tile != kTile) return DWARF_ERR_SHAPE;
  if (a->B < 0 || a->H <= 0 || a->T < 0 || a->C < 1 || a->k_slots < 0 || a->k_slots > kTopK) return DWARF_ERR_SHAPE;
  if (a->B == 0 || a->T == 0) return DWARF_OK;
  if (!a->query || !a->reps || !a->top_chunk_idx || !a->route_scale || !a->route) return DWARF_ERR_NULL;
  if (!al16(a->query) || (a->sqb | a->sqh | a->sqn) % 8 || (reinterpret_cast<uintptr_t>(a->route) & 7u))
    return DWARF_ERR_ALIGN;
  RouteParams p{};
  p.q = (const __nv_bfloat16*)a->query; p.sqb = a->sqb; p.sqh = a->sqh; p.sqn = a->sqn;
  p.reps = (const __nv_bfloat16*)a->reps; p.top = a->top_chunk_idx; p.route_scale = a->route_scale;
  p.route = (__nv_bfloat16*)a->route;
  p.H = a->H; p.T = a->T; p.C = a->C; p.tiles = (a->T + kTile - 1) / kTile; p.k_slots = a->k_slots;
  int64_t n_tiles = 0;
  if (!launch_window(a->tile_begin, a->tile_count, a->pos, &p, &n_tiles)) return DWARF_ERR_SHAPE;
  if (n_tiles == 0) return DWARF_OK;
  dim3 grid((unsigned)((n_tiles + 7) / 8), (unsigned)a->H, (unsigned)a->B);
  hisa_route_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(p);
  return launch_status();
}

extern "C" int dwarf_hisa_attn(const dwarf_hisa_attn_args* a, void* stream) {
  DWARF_CHECK_VERSION(a);
  if (a->head_dim != kHD || a->chunk_size != kChunk || a->selector_tile != kTile || a->local_window != kWindow)
    return DWARF_ERR_SHAPE;
  if (a->B < 0 || a->H <= 0 || a->T < 0 || a->k_slots < 0 || a->k_slots > kTopK) return DWARF_ERR_SHAPE;
  if (a->B == 0 || a->T == 0) return DWARF_OK;
  if (!a->query || !a->local_key || !a->local_value || !a->global_key || !a->global_value || !a->route ||
      !a->top_chunk_idx || !a->lengths || !a->out)
    return DWARF_ERR_NULL;
  const void* rows[] = {a->query, a->local_key, a->local_value, a->global_key, a->global_value, a->out};
  for (const void* r : rows)
    if (!al16(r)) return DWARF_ERR_ALIGN;
  const int64_t strides[] = {a->sqb, a->sqh, a->sqn, a->slkb, a->slkh, a->slkn, a->slvb, a->slvh, a->slvn,
                             a->sgkb, a->sgkh, a->sgkn, a->sgvb, a->sgvh, a->sgvn, a->sob, a->soh, a->son};
  for (int64_t s : strides)
    if (s % 8 != 0) return DWARF_ERR_ALIGN;
  if (a->T > 0x7fffffffLL) return DWARF_ERR_SHAPE;
  AttnParams p{};
  p.q = (const __nv_bfloat16*)a->query; p.sqb = a->sqb; p.sqh = a->sqh; p.sqn = a->sqn;
  p.lk = (const __nv_bfloat16*)a->local_key; p.slkb = a->slkb; p.slkh = a->slkh; p.slkn = a->slkn;
  p.lv = (const __nv_bfloat16*)a->local_value; p.slvb = a->slvb; p.slvh = a->slvh; p.slvn = a->slvn;
  p.gk = (const __nv_bfloat16*)a->global_key; p.sgkb = a->sgkb; p.sgkh = a->sgkh; p.sgkn = a->sgkn;
  p.gv = (const __nv_bfloat16*)a->global_value; p.sgvb = a->sgvb; p.sgvh = a->sgvh; p.sgvn = a->sgvn;
  p.top = a->top_chunk_idx; p.route = (const __nv_bfloat16*)a->route;
  p.lengths = a->lengths;
  p.out = (__nv_bfloat16*)a->out; p.sob = a->sob; p.soh = a->soh; p.son = a->son;
  p.lse = (float*)a->lse;
  p.H = a->H; p.T = a->T; p.tiles = (a->T + kTile - 1) / kTile;
  p.k_slots = a->k_slots;
  TcMaps maps;
  if (!make_kv_map(&maps.lk, a->local_key, a->B, a->H, a->T, a->slkb, a->slkh, a->slkn) ||
      !make_kv_map(&maps.lv, a->local_value, a->B, a->H, a->T, a->slvb, a->slvh, a->slvn) ||
      !make_kv_map(&maps.gk, a->global_key, a->B, a->H, a->T, a->sgkb, a->sgkh, a->sgkn) ||
      !make_kv_map(&maps.gv, a->global_value, a->B, a->H, a->T, a->sgvb, a->sgvh, a->sgvn) ||
      !make_kv_map(&maps.q, a->query, a->B, a->H, a->T, a->sqb, a->sqh, a->sqn))
    return DWARF_ERR_LAUNCH;
  // The tensor-core kernel by default; DWARF_HISA_ATTN=mma selects the mma.sync
  // form (read on every call).
  const char* which = getenv("DWARF_HISA_ATTN");
  const bool tc = !(which != nullptr && which[0] == 'm');
  const size_t smem = tc ? (size_t)TcSmem::bytes : (size_t)AttnSmem::bytes;
  if (cudaFuncSetAttribute(tc ? (const void*)hisa_attn_tc_kernel : (const void*)hisa_attn_kernel,
                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return DWARF_ERR_LAUNCH;
  const int64_t cta_tiles = kCtaTiles;
  int64_t n_tiles = 0;
  if (!launch_window(a->tile_begin, a->tile_count, a->pos, &p, &n_tiles)) return DWARF_ERR_SHAPE;
  if (n_tiles == 0) return DWARF_OK;
  p.grid_begin = p.tile_begin - p.tile_begin % cta_tiles;
  // A device window may straddle a CTA group boundary: one spare CTA (it exits at once).
  const int64_t ctas = a->pos != nullptr ? (n_tiles == 1 ? 1 : (n_tiles + cta_tiles - 1) / cta_tiles + 1)
                                         : (p.tile_end - p.grid_begin + cta_tiles - 1) / cta_tiles;
  dim3 grid((unsigned)ctas, (unsigned)a->H, (unsigned)a->B);
  if (tc) {
    hisa_attn_tc_kernel<<<grid, kTcThreads, smem, (cudaStream_t)stream>>>(p, maps, a->device_status);
  } else {
    const AttnMaps m4{maps.lk, maps.lv, maps.gk, maps.gv};
    hisa_attn_kernel<<<grid, kCtaTiles * 32, smem, (cudaStream_t)stream>>>(p, m4, a->device_status);
  }
  return launch_status();
}
