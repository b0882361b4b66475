// Backward of the HISA fused tile attention (hisa.cu, hisa_attn_kernel): the
// gradients of the reference's local lane + global lane + exact LSE merge
// (kernels/hierarchical_sparse_attn_v18_hisa.py:688-835, 1103-1246, 1982-2027).
//
// With P the joint softmax of a query over its local window (keys n-64..n-1 of
// local K/V) and its tile's routed chunks (keys of global K/V with id < n-64,
// score + the slot's route prior), dP = dO . v, delta = dO . O, dS = P (dP - delta):
//   dq = (1/8) sum dS k,  dk = (1/8) sum dS q,  dv = sum P dO,
//   d_route[n, slot] = sum of dS over the slot's chunk.
// All products run on bf16 tensor cores (mma.sync m16n8k16, fp32 accumulate),
// the structure of a FlashAttention-2 backward:
//  1. query side, one warp per 16-query selector tile (4 per CTA): with the row
//     lse the forward launch stored (log2 domain), it forms P, dP, dS over the
//     tile's key blocks of 16 (a three-stage cp.async pipeline) and accumulates
//     dq (dS in bf16 times K) and d_route; it stores each row's delta for step 2;
//  2. key side, one CTA per 64 key rows (4 warps x 16 keys), separately for the
//     local K/V (query tiles of the rows' windows) and the global K/V (the tiles
//     that routed the chunk, found by scanning top_chunk_idx): S^T = K Q^T from
//     the stored lse gives P^T and dS^T, then dV = P^T dO and dK = dS^T Q.
// Every gradient row has one writer: no atomics, no zero-fill, and repeated
// runs are bit-identical.
#include "common.cuh"
#include "warp_mma.cuh"

namespace dwarf {
namespace {
using namespace wmma16;

constexpr int kBT = 16;        // queries per selector tile
constexpr int kBChunk = 64;    // chunk rows == key rows per key-side CTA
constexpr int kBWindow = 64;
constexpr int kBSlots = 4;
constexpr int kBWarps = 4;
constexpr int kBStages = 3;  // query-side key-block pipeline depth
constexpr float kBScale = 0.125f;
constexpr float kBLog2e = 1.4426950408889634f;

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// A fragments (m16n8k16, row-major 16 x 64) of rows r0..r0+15 of a contiguous
// [T][64] bf16 matrix; rows outside [0, T) read row 0 (their products are masked).
__device__ __forceinline__ void load_a(const __nv_bfloat16* m, int64_t r0, int64_t T, int lane, uint32_t (&a)[4][4]) {
  const int g = lane >> 2, t4 = lane & 3;
  int64_t ra = r0 + g, rb = r0 + g + 8;
  ra = (ra >= 0 && ra < T) ? ra : 0;
  rb = (rb >= 0 && rb < T) ? rb : 0;
#pragma unroll
  for (int kt = 0; kt < 4; ++kt) {
    const int c0 = kt * 16 + 2 * t4;
    a[kt][0] = *reinterpret_cast<const uint32_t*>(m + ra * 64 + c0);
    a[kt][1] = *reinterpret_cast<const uint32_t*>(m + rb * 64 + c0);
    a[kt][2] = *reinterpret_cast<const uint32_t*>(m + ra * 64 + c0 + 8);
    a[kt][3] = *reinterpret_cast<const uint32_t*>(m + rb * 64 + c0 + 8);
  }
}

// 16 rows r0.. of a contiguous [T][64] bf16 matrix -> swizzled smem tile (zero
// rows outside [0, T)); called by the 32 lanes of one warp or by `nthreads` threads.
__device__ __forceinline__ void stage16(uint32_t tile, const __nv_bfloat16* m, int64_t r0, int64_t T, int tid,
                                        int nthreads) {
  for (int i = tid; i < 16 * 8; i += nthreads) {
    const int r = i >> 3, c = i & 7;
    const int64_t row = r0 + r;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (row >= 0 && row < T) v = *reinterpret_cast<const uint4*>(m + row * 64 + c * 8);
    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(tile_addr(tile, r, c)), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w) : "memory");
  }
}

// stage16 through cp.async (16-byte copies, zero-filled outside [0, T)); the
// caller commits and waits.
__device__ __forceinline__ void stage16_async(uint32_t tile, const __nv_bfloat16* m, int64_t r0, int64_t T, int tid,
                                              int nthreads) {
  for (int i = tid; i < 16 * 8; i += nthreads) {
    const int r = i >> 3, c = i & 7;
    const int64_t row = r0 + r;
    const bool ok = row >= 0 && row < T;
    const __nv_bfloat16* src = m + (ok ? row : 0) * 64 + c * 8;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(tile_addr(tile, r, c)), "l"(src),
                 "r"(ok ? 16 : 0) : "memory");
  }
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// C[16 x 16] = A[16 x 64] . M^T for the 16-row smem tile M (rows = the n index).
__device__ __forceinline__ void mma_abt(const uint32_t (&a)[4][4], uint32_t tile, int lane, float (&c)[2][4]) {
#pragma unroll
  for (int j = 0; j < 2; ++j) c[j][0] = c[j][1] = c[j][2] = c[j][3] = 0.0f;
  const int mtx = lane >> 3, r = lane & 7;
#pragma unroll
  for (int kt = 0; kt < 4; ++kt) {
    uint32_t b0, b1, b2, b3;
    ldsm_x4(tile_addr(tile, (mtx >> 1) * 8 + r, kt * 2 + (mtx & 1)), b0, b1, b2, b3);
    mma_bf16(c[0], a[kt], b0, b1);
    mma_bf16(c[1], a[kt], b2, b3);
  }
}

// acc[16 x 64] += P[16 x 16] . M for the 16-row smem tile M (rows = the k index);
// P comes as the bf16 A fragment built from a 16 x 16 accumulator pair.
__device__ __forceinline__ void mma_pm(const uint32_t (&pa)[4], uint32_t tile, int lane, float (&acc)[8][4]) {
  const int mtx = lane >> 3, r = lane & 7;
#pragma unroll
  for (int n = 0; n < 8; n += 2) {
    uint32_t b0, b1, b2, b3;
    ldsm_x4_t(tile_addr(tile, (mtx & 1) * 8 + r, n + (mtx >> 1)), b0, b1, b2, b3);
    mma_bf16(acc[n], pa, b0, b1);
    mma_bf16(acc[n + 1], pa, b2, b3);
  }
}

__device__ __forceinline__ void a_from_acc(const float (&c)[2][4], uint32_t (&pa)[4]) {
  pa[0] = pack2(c[0][0], c[0][1]);
  pa[1] = pack2(c[0][2], c[0][3]);
  pa[2] = pack2(c[1][0], c[1][1]);
  pa[3] = pack2(c[1][2], c[1][3]);
}

struct BwdParams {
  const __nv_bfloat16 *q, *lk, *lv, *gk, *gv, *out, *dout, *route;
  const int32_t *top, *lengths;
  float *dq, *dlk, *dlv, *dgk, *dgv, *droute, *delta;
  const float* lse;  // the forward's row lse (log2 domain)
  int64_t H, T, tiles;
  int k_slots;
};

// ---------------------------------------------------------------- 1. query side
// Key block kb of a tile: kb < 5 local blocks of 16 rows from t0 - 64, then
// 4 blocks per routed slot.
__global__ void __launch_bounds__(kBWarps * 32) hisa_bwd_query_kernel(const BwdParams p) {
  __shared__ __align__(128) unsigned char s_kv[kBWarps][kBStages][2][16 * 128];  // [warp][stage][K, V]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int64_t h = blockIdx.y, b = blockIdx.z;
  const int64_t t = (int64_t)blockIdx.x * kBWarps + warp;
  if (t >= p.tiles) return;  // warp-uniform; no CTA-wide barrier below
  const int64_t T = p.T, t0 = t * kBT;
  const int64_t len = p.lengths[b] < T ? p.lengths[b] : T;
  const int64_t bh = (b * p.H + h) * T;
  const uint32_t kv0 = smem_u32(s_kv[warp][0][0]);  // buffer x: K at kv0 + x * 4096, V 2048 above
  int slot_chunk[kBSlots];
  {
    const int32_t* top = p.top + ((b * p.H + h) * p.tiles + t) * p.k_slots;
#pragma unroll
    for (int s = 0; s < kBSlots; ++s) slot_chunk[s] = s < p.k_slots ? top[s] : -1;
  }
  uint32_t qa[4][4], ga[4][4];
  load_a(p.q + bh * 64, t0, T, lane, qa);
  load_a(p.dout + bh * 64, t0, T, lane, ga);
  // delta = dO . O per row (rows g and g + 8 of the tile), fp32 of the bf16 values
  float delta[2], route[2][kBSlots];
  {
    uint32_t oa[4][4];
    load_a(p.out + bh * 64, t0, T, lane, oa);
    delta[0] = delta[1] = 0.0f;
#pragma unroll
    for (int kt = 0; kt < 4; ++kt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float d = bf_lo(ga[kt][i]) * bf_lo(oa[kt][i]) + bf_hi(ga[kt][i]) * bf_hi(oa[kt][i]);
        delta[i & 1] += d;
      }
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      delta[rr] += __shfl_xor_sync(0xffffffffu, delta[rr], 1);
      delta[rr] += __shfl_xor_sync(0xffffffffu, delta[rr], 2);
      const int64_t n = t0 + g + 8 * rr;
#pragma unroll
      for (int s = 0; s < kBSlots; ++s)
        route[rr][s] = (n < T && s < p.k_slots) ? __bfloat162float(p.route[(bh + n) * kBSlots + s]) : 0.0f;
    }
  }
  const int n_blocks = 5 + 4 * kBSlots;
  // key block -> (first row, slot or -1); false when the block does not exist
  auto block = [&](int kb, int64_t& r0, int& slot) -> bool {
    if (kb < 5) {
      r0 = t0 - kBWindow + 16 * kb;
      slot = -1;
      return r0 + 16 > 0 && r0 < T;
    }
    slot = (kb - 5) >> 2;
    int c = -1;
#pragma unroll
    for (int q = 0; q < kBSlots; ++q) c = q == slot ? slot_chunk[q] : c;
    r0 = (int64_t)c * kBChunk + 16 * ((kb - 5) & 3);
    return c >= 0 && r0 < T;
  };
  // log2-domain scores of the block for rows g, g + 8 (-inf where masked);
  // 32-bit positions (T <= 8192)
  const int ti = (int)t0, leni = (int)len;
  auto scores = [&](float (&s)[2][4], int r0, int slot) {
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int rr = e >> 1;
        const int n = ti + g + 8 * rr, k = r0 + j * 8 + 2 * t4 + (e & 1);
        const bool ok = n < leni && k >= 0 && (slot < 0 ? (k < n && k >= n - kBWindow) : (k < n - kBWindow && k < leni));
        float bias = 0.0f;
#pragma unroll
        for (int q = 0; q < kBSlots; ++q) bias = q == slot ? route[rr][q] : bias;  // register select
        s[j][e] = ok ? (s[j][e] * kBScale + bias) * kBLog2e : -INFINITY;
      }
  };
  // Row lse (log2 domain) from the forward launch.
  float lse[2];
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int64_t n = t0 + g + 8 * rr;
    lse[rr] = n < T ? p.lse[bh + n] : INFINITY;
  }
  // Three-stage cp.async pipeline over the 21 key-block positions (absent blocks
  // issue nothing and compute nothing): block kb uses buffer kb % 3, and the
  // copies of blocks kb + 1 and kb + 2 are in flight while kb is computed.
  auto issue = [&](int kb) {
    int64_t r0;
    int slot;
    if (!block(kb, r0, slot)) return;
    const uint32_t kt = kv0 + (kb % kBStages) * 4096;
    stage16_async(kt, (slot < 0 ? p.lk : p.gk) + bh * 64, r0, T, lane, 32);
    stage16_async(kt + 2048, (slot < 0 ? p.lv : p.gv) + bh * 64, r0, T, lane, 32);
  };
  float dq[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n) dq[n][0] = dq[n][1] = dq[n][2] = dq[n][3] = 0.0f;
  float droute[2][kBSlots];
#pragma unroll
  for (int rr = 0; rr < 2; ++rr)
#pragma unroll
    for (int q = 0; q < kBSlots; ++q) droute[rr][q] = 0.0f;
  issue(0);
  cp_commit();
  issue(1);
  cp_commit();
  for (int kb = 0; kb < n_blocks; ++kb) {
    if (kb + 2 < n_blocks) issue(kb + 2);
    cp_commit();
    cp_wait<2>();
    __syncwarp();
    int64_t r0l;
    int slot;
    if (block(kb, r0l, slot)) {  // warp-uniform
      const uint32_t ktile = kv0 + (kb % kBStages) * 4096, vtile = ktile + 2048;
      float s[2][4], dp[2][4];
      mma_abt(qa, ktile, lane, s);
      scores(s, (int)r0l, slot);
      mma_abt(ga, vtile, lane, dp);
      float rsum[2] = {0.0f, 0.0f};
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int rr = e >> 1;
          const float pr = ex2_approx(s[j][e] - lse[rr]);
          const float ds = pr * (dp[j][e] - delta[rr]);
          s[j][e] = ds;
          rsum[rr] += ds;
        }
      uint32_t pa[4];
      a_from_acc(s, pa);
      mma_pm(pa, ktile, lane, dq);
#pragma unroll
      for (int q = 0; q < kBSlots; ++q)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) droute[rr][q] += q == slot ? rsum[rr] : 0.0f;
    }
    __syncwarp();  // buffer kb % 3 is refilled by the issue of the next iteration
  }
  // ---- stores: dq, d_route (rows g, g + 8), delta for the key side
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int64_t n = t0 + g + 8 * rr;
#pragma unroll
    for (int s = 0; s < kBSlots; ++s) {
      droute[rr][s] += __shfl_xor_sync(0xffffffffu, droute[rr][s], 1);
      droute[rr][s] += __shfl_xor_sync(0xffffffffu, droute[rr][s], 2);
    }
    if (n < T) {
#pragma unroll
      for (int nn = 0; nn < 8; ++nn)
        *reinterpret_cast<float2*>(p.dq + (bh + n) * 64 + nn * 8 + 2 * t4) =
            make_float2(dq[nn][2 * rr] * kBScale, dq[nn][2 * rr + 1] * kBScale);
      if (t4 == 0) {
        *reinterpret_cast<float4*>(p.droute + (bh + n) * kBSlots) =
            make_float4(droute[rr][0], droute[rr][1], droute[rr][2], droute[rr][3]);
        p.delta[bh + n] = delta[rr];
      }
    }
  }
}

// ---------------------------------------------------------------- 2. key side
// CTA = 64 key rows [k0, k0 + 64) of one (b, h); warp w owns rows k0 + 16 w ...
// GLOBAL = false: local K/V, query tiles whose windows reach the rows;
// GLOBAL = true: global K/V rows of chunk k0 / 64, query tiles that routed it.
constexpr int kBMaxTiles = 512;  // T <= 8192 (128 chunks): at most 512 selector tiles

template <bool GLOBAL>
__global__ void __launch_bounds__(kBWarps * 32) hisa_bwd_key_kernel(const BwdParams p) {
  __shared__ __align__(128) unsigned char s_tile[2][2][16 * 128];  // [buffer][Q, dO] of a query tile
  __shared__ float s_lse[2][16], s_delta[2][16], s_bias[2][16];
  __shared__ int16_t s_list[kBMaxTiles];
  __shared__ int8_t s_slot[kBMaxTiles];
  __shared__ int s_count;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int64_t h = blockIdx.y, b = blockIdx.z;
  const int64_t T = p.T, k0 = (int64_t)blockIdx.x * kBChunk;
  const int64_t len = p.lengths[b] < T ? p.lengths[b] : T;
  const int64_t bh = (b * p.H + h) * T;
  const uint32_t tiles0 = smem_u32(s_tile[0][0]);  // buffer x: Q at tiles0 + x * 4096, dO 2048 above

  // ---- the query tiles that see these rows
  if (GLOBAL) {
    if (tid == 0) s_count = 0;
    __syncthreads();
    const int c = (int)blockIdx.x;
    const int32_t* top = p.top + (b * p.H + h) * p.tiles * p.k_slots;
    // tiles in ascending order: each warp takes 32 consecutive tiles per pass
    for (int64_t base = 0; base < p.tiles; base += kBWarps * 32) {
      const int64_t t = base + tid;
      int slot = -1;
      if (t < p.tiles)
        for (int q = 0; q < p.k_slots; ++q) slot = top[t * p.k_slots + q] == c ? q : slot;
      // a chunk is routed at most once per tile; tiles starting before the
      // chunk's end + 64 have no query that may use it (ids < n - 64)
      const bool hit = slot >= 0 && t * kBT + kBT - 1 - kBWindow > k0;
      const unsigned mask = __ballot_sync(0xffffffffu, hit);
      __shared__ int s_warp_n[kBWarps];
      if (lane == 0) s_warp_n[warp] = __popc(mask);
      __syncthreads();
      int before = s_count;
      for (int w = 0; w < warp; ++w) before += s_warp_n[w];
      if (hit) {
        const int at = before + __popc(mask & ((1u << lane) - 1u));
        s_list[at] = (int16_t)t;
        s_slot[at] = (int8_t)slot;
      }
      __syncthreads();
      if (tid == 0) for (int w = 0; w < kBWarps; ++w) s_count += s_warp_n[w];
      __syncthreads();
    }
  } else {
    // queries n in [k0 + 1, k0 + 64 + 63] see some row of [k0, k0 + 64)
    if (tid == 0) {
      const int64_t t_first = (k0 + 1) / kBT;
      int64_t t_last = (k0 + kBChunk - 1 + kBWindow) / kBT;
      if (t_last > p.tiles - 1) t_last = p.tiles - 1;
      int n = 0;
      for (int64_t t = t_first; t <= t_last; ++t) {
        s_list[n] = (int16_t)t;
        s_slot[n] = -1;
        ++n;
      }
      s_count = n;
    }
    __syncthreads();
  }
  const int n_tiles = s_count;

  // ---- this warp's 16 key rows as A fragments (K and V)
  const int64_t r0 = k0 + 16 * warp;
  const __nv_bfloat16* kmat = (GLOBAL ? p.gk : p.lk) + bh * 64;
  const __nv_bfloat16* vmat = (GLOBAL ? p.gv : p.lv) + bh * 64;
  uint32_t ka[4][4], va[4][4];
  load_a(kmat, r0, T, lane, ka);
  load_a(vmat, r0, T, lane, va);
  float dk[8][4], dv[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n) dk[n][0] = dk[n][1] = dk[n][2] = dk[n][3] = dv[n][0] = dv[n][1] = dv[n][2] = dv[n][3] = 0.0f;

  // Double-buffered: tile i + 1's Q / dO copies (cp.async) and its per-row lse,
  // delta and route prior (registers of threads 0..15) load while tile i computes.
  float nl = INFINITY, nd = 0.0f, nb = 0.0f;
  auto issue = [&](int i, int buf) {
    const int64_t t0 = (int64_t)s_list[i] * kBT;
    const int slot = s_slot[i];
    stage16_async(tiles0 + buf * 4096, p.q + bh * 64, t0, T, tid, kBWarps * 32);
    stage16_async(tiles0 + buf * 4096 + 2048, p.dout + bh * 64, t0, T, tid, kBWarps * 32);
    if (tid < 16) {
      const int64_t n = t0 + tid;
      const bool ok = n < T;
      nl = ok ? p.lse[bh + n] : INFINITY;
      nd = ok ? p.delta[bh + n] : 0.0f;
      nb = (ok && slot >= 0) ? __bfloat162float(p.route[(bh + n) * kBSlots + slot]) : 0.0f;
    }
  };
  if (n_tiles > 0) issue(0, 0);
  cp_commit();
  for (int i = 0; i < n_tiles; ++i) {
    const int buf = i & 1;
    const int64_t t0 = (int64_t)s_list[i] * kBT;
    if (tid < 16) {
      s_lse[buf][tid] = nl;
      s_delta[buf][tid] = nd;
      s_bias[buf][tid] = nb;
    }
    if (i + 1 < n_tiles) issue(i + 1, buf ^ 1);
    cp_commit();
    cp_wait<1>();
    __syncthreads();  // tile i visible to every warp
    const uint32_t qtile = tiles0 + buf * 4096, gtile = qtile + 2048;
    const float* s_lse_b = s_lse[buf];
    const float* s_delta_b = s_delta[buf];
    const float* s_bias_b = s_bias[buf];
    // S^T [16 keys x 16 queries], dP^T likewise
    float s[2][4], dp[2][4];
    mma_abt(ka, qtile, lane, s);
    mma_abt(va, gtile, lane, dp);
    float ds[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int64_t k = r0 + g + 8 * (e >> 1);
        const int qi = j * 8 + 2 * t4 + (e & 1);
        const int64_t n = t0 + qi;
        const bool ok = n < len && k < T &&
                        (GLOBAL ? (k < n - kBWindow && k < len) : (k < n && k >= n - kBWindow));
        const float x = ok ? (s[j][e] * kBScale + s_bias_b[qi]) * kBLog2e : -INFINITY;
        const float pr = ex2_approx(x - s_lse_b[qi]);
        s[j][e] = pr;
        ds[j][e] = pr * (dp[j][e] - s_delta_b[qi]);
      }
    uint32_t pa[4], da[4];
    a_from_acc(s, pa);
    a_from_acc(ds, da);
    mma_pm(pa, gtile, lane, dv);  // dV += P^T dO
    mma_pm(da, qtile, lane, dk);  // dK += dS^T Q
    __syncthreads();  // buffer buf is refilled by the next iteration's issue
  }
  // ---- one writer per row
  float* dkm = (GLOBAL ? p.dgk : p.dlk) + bh * 64;
  float* dvm = (GLOBAL ? p.dgv : p.dlv) + bh * 64;
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int64_t k = r0 + g + 8 * rr;
    if (k >= T) continue;
#pragma unroll
    for (int nn = 0; nn < 8; ++nn) {
      *reinterpret_cast<float2*>(dkm + k * 64 + nn * 8 + 2 * t4) =
          make_float2(dk[nn][2 * rr] * kBScale, dk[nn][2 * rr + 1] * kBScale);
      *reinterpret_cast<float2*>(dvm + k * 64 + nn * 8 + 2 * t4) = make_float2(dv[nn][2 * rr], dv[nn][2 * rr + 1]);
    }
  }
}

}  // namespace
}  // namespace dwarf

using namespace dwarf;

extern "C" int dwarf_hisa_attn_bwd(const dwarf_hisa_attn_bwd_args* a, void* stream) {
  DWARF_CHECK_VERSION(a);
  if (a->B < 0 || a->H <= 0 || a->T < 0 || a->k_slots < 0 || a->k_slots > kBSlots) return DWARF_ERR_SHAPE;
  if (a->B > 65535 || a->H > 65535 || a->T > (int64_t)kBMaxTiles * kBT) return DWARF_ERR_SHAPE;
  if (a->B == 0 || a->T == 0) return DWARF_OK;
  if (!a->query || !a->local_key || !a->local_value || !a->global_key || !a->global_value || !a->route ||
      !a->lengths || !a->out || !a->dout || !a->dq || !a->d_local_key || !a->d_local_value ||
      !a->d_global_key || !a->d_global_value || !a->d_route || !a->lse || !a->delta ||
      (a->k_slots > 0 && !a->top_chunk_idx))
    return DWARF_ERR_NULL;
  const void* rows[] = {a->query, a->local_key, a->local_value, a->global_key, a->global_value, a->out, a->dout,
                        a->dq, a->d_local_key, a->d_local_value, a->d_global_key, a->d_global_value, a->d_route};
  for (const void* r : rows)
    if (!aligned16(r)) return DWARF_ERR_ALIGN;
  if (reinterpret_cast<uintptr_t>(a->route) & 7u) return DWARF_ERR_ALIGN;
  BwdParams p;
  p.q = (const __nv_bfloat16*)a->query; p.lk = (const __nv_bfloat16*)a->local_key;
  p.lv = (const __nv_bfloat16*)a->local_value; p.gk = (const __nv_bfloat16*)a->global_key;
  p.gv = (const __nv_bfloat16*)a->global_value; p.out = (const __nv_bfloat16*)a->out;
  p.dout = (const __nv_bfloat16*)a->dout; p.route = (const __nv_bfloat16*)a->route;
  p.top = a->top_chunk_idx; p.lengths = a->lengths;
  p.dq = a->dq; p.dlk = a->d_local_key; p.dlv = a->d_local_value; p.dgk = a->d_global_key;
  p.dgv = a->d_global_value; p.droute = a->d_route; p.lse = a->lse; p.delta = a->delta;
  p.H = a->H; p.T = a->T; p.tiles = (a->T + kBT - 1) / kBT; p.k_slots = a->k_slots;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  hisa_bwd_query_kernel<<<dim3((unsigned)((p.tiles + kBWarps - 1) / kBWarps), (unsigned)a->H, (unsigned)a->B),
                          kBWarps * 32, 0, st>>>(p);
  const unsigned blocks = (unsigned)((a->T + kBChunk - 1) / kBChunk);
  hisa_bwd_key_kernel<false><<<dim3(blocks, (unsigned)a->H, (unsigned)a->B), kBWarps * 32, 0, st>>>(p);
  hisa_bwd_key_kernel<true><<<dim3(blocks, (unsigned)a->H, (unsigned)a->B), kBWarps * 32, 0, st>>>(p);
  return launch_status();
}
