// Backward of the HISA fused tile attention (hisa.cu, hisa_attn_kernel): the
// gradients of the reference's local lane + global lane + exact LSE merge
// (kernels/hierarchical_sparse_attn_v18_hisa.py:688-835, 1103-1246, 1982-2027).
//
// One CTA of 256 threads per (b, h, 16-query selector tile). The tile's key
// set is dense: the local window rows [t0 - 64, t0 + 15) of (local_key,
// local_value) and the 64 rows of each routed chunk of (global_key,
// global_value). Keys go through shared memory in blocks of 32 (fp32, rows
// padded to 65 floats so the per-key dot products are bank-conflict-free):
// pass 1 recomputes each query's lse (online max / sum), pass 2 forms P, dP,
// dS and accumulates dq in registers, d_route per slot, and the block's dK/dV
// rows, which are added to the fp32 gradient buffers with float4 atomics.
#include "common.cuh"

namespace dwarf {
namespace {

constexpr int kHT = 256;       // threads
constexpr int kHQ = 16;        // queries per tile
constexpr int kHKB = 32;       // keys per block
constexpr int kHChunk = 64;
constexpr int kHWindow = 64;
constexpr int kHLd = 65;       // padded row length (floats)
constexpr int kHMaxBlocks = 3 + 2 * 4;
constexpr float kHScale = 0.125f;

struct KeyBlock {
  int64_t row0;
  int rows;
  int slot;  // -1: local window block, else the routed slot
};

__device__ __forceinline__ float half_warp_sum(float x) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}
__device__ __forceinline__ float half_warp_max(float x) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

// `rows` x 64 bf16 rows of src (row stride 64) -> fp32 dst[CAP][kHLd]; zero past `rows`.
template <int CAP>
__device__ __forceinline__ void stage_rows(float (*dst)[kHLd], const __nv_bfloat16* src, int rows, int tid) {
  for (int i = tid; i < CAP * 16; i += kHT) {
    const int r = i >> 4, c = (i & 15) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < rows) {
      const uint2 w = *reinterpret_cast<const uint2*>(src + (int64_t)r * 64 + c);
      v = make_float4(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xffff0000u),
                      __uint_as_float(w.y << 16), __uint_as_float(w.y & 0xffff0000u));
    }
    dst[r][c] = v.x; dst[r][c + 1] = v.y; dst[r][c + 2] = v.z; dst[r][c + 3] = v.w;
  }
}

__global__ void __launch_bounds__(kHT) hisa_attn_bwd_kernel(const dwarf_hisa_attn_bwd_args a) {
  __shared__ float sQ[kHQ][kHLd], sdO[kHQ][kHLd];
  __shared__ float sK[kHKB][kHLd], sV[kHKB][kHLd];
  __shared__ float sP[kHQ][kHKB + 1], sdS[kHQ][kHKB + 1];
  __shared__ float s_delta[kHQ], s_route[kHQ][4], s_droute[kHQ][4];
  __shared__ KeyBlock s_blk[kHMaxBlocks];
  __shared__ int s_nblk;

  const int tid = threadIdx.x;
  const int64_t t = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int64_t T = a.T;
  const int64_t n0 = t * kHQ;
  const int64_t len = a.lengths[b] < T ? a.lengths[b] : T;
  const int64_t bh = (b * a.H + h) * T;
  const __nv_bfloat16* Q = static_cast<const __nv_bfloat16*>(a.query) + bh * 64;
  const __nv_bfloat16* LK = static_cast<const __nv_bfloat16*>(a.local_key) + bh * 64;
  const __nv_bfloat16* LV = static_cast<const __nv_bfloat16*>(a.local_value) + bh * 64;
  const __nv_bfloat16* GK = static_cast<const __nv_bfloat16*>(a.global_key) + bh * 64;
  const __nv_bfloat16* GV = static_cast<const __nv_bfloat16*>(a.global_value) + bh * 64;
  const int nq = (int)(T - n0 < kHQ ? T - n0 : kHQ);

  // ---- tile inputs: Q, dO (fp32), delta = dO . O, route, block list
  stage_rows<kHQ>(sQ, Q + n0 * 64, nq, tid);
  __syncthreads();
  {
    const int qi = tid >> 4, d4 = (tid & 15) * 4;
    const int64_t n = n0 + qi;
    float dsum = 0.f;
    float o[4] = {0.f, 0.f, 0.f, 0.f}, g[4] = {0.f, 0.f, 0.f, 0.f};
    if (qi < nq) {
      const uint2 wo = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(a.out) + (bh + n) * 64 + d4);
      const uint2 wg = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(a.dout) + (bh + n) * 64 + d4);
      o[0] = __uint_as_float(wo.x << 16); o[1] = __uint_as_float(wo.x & 0xffff0000u);
      o[2] = __uint_as_float(wo.y << 16); o[3] = __uint_as_float(wo.y & 0xffff0000u);
      g[0] = __uint_as_float(wg.x << 16); g[1] = __uint_as_float(wg.x & 0xffff0000u);
      g[2] = __uint_as_float(wg.y << 16); g[3] = __uint_as_float(wg.y & 0xffff0000u);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      dsum = fmaf(g[i], o[i], dsum);
      sdO[qi][d4 + i] = g[i];
    }
    dsum = half_warp_sum(dsum);
    if ((tid & 15) == 0) s_delta[qi] = dsum;
    if (tid < kHQ * 4) {
      const int q = tid >> 2, k = tid & 3;
      float r = 0.f;
      if (q < nq && k < a.k_slots)
        r = __bfloat162float(static_cast<const __nv_bfloat16*>(a.route)[(bh + n0 + q) * 4 + k]);
      s_route[q][k] = r;
      s_droute[q][k] = 0.f;
    }
    if (tid == 0) {
      int nb = 0;
      const int64_t lo = n0 - kHWindow > 0 ? n0 - kHWindow : 0;
      const int64_t hi = n0 + nq - 1;  // exclusive: the last query's last local key is hi - 1
      for (int64_t r = lo; r < hi; r += kHKB) s_blk[nb++] = KeyBlock{r, (int)(hi - r < kHKB ? hi - r : kHKB), -1};
      const int32_t* top = a.top_chunk_idx + ((b * a.H + h) * ((T + kHQ - 1) / kHQ) + t) * a.k_slots;
      for (int k = 0; k < a.k_slots; ++k) {
        const int c = top[k];
        if (c < 0) continue;
        for (int64_t r = (int64_t)c * kHChunk; r < (int64_t)(c + 1) * kHChunk && r < T; r += kHKB) {
          const int64_t end = (int64_t)(c + 1) * kHChunk < T ? (int64_t)(c + 1) * kHChunk : T;
          s_blk[nb++] = KeyBlock{r, (int)(end - r < kHKB ? end - r : kHKB), k};
        }
      }
      s_nblk = nb;
    }
  }
  __syncthreads();

  // Score thread layout: query qi = tid / 16 (a half warp per query), keys kk, kk + 1.
  const int qi = tid >> 4, kk = (tid & 15) * 2;
  const int64_t n = n0 + qi;
  const bool qvalid = qi < nq && n < len;
  auto score = [&](const KeyBlock& blk, int e, float& s, bool& ok) {
    const int k = kk + e;
    const int64_t r = blk.row0 + k;
    float acc = 0.f;
#pragma unroll 16
    for (int d = 0; d < 64; ++d) acc = fmaf(sQ[qi][d], sK[k][d], acc);
    if (blk.slot < 0) ok = qvalid && k < blk.rows && r < n && r >= n - kHWindow;
    else ok = qvalid && k < blk.rows && r < n - kHWindow && r < len;
    s = blk.slot < 0 ? acc * kHScale : fmaf(acc, kHScale, s_route[qi][blk.slot]);
  };

  // ---- pass 1: lse per query
  float m = -INFINITY, l = 0.f;
  const int nblk = s_nblk;
  for (int bi = 0; bi < nblk; ++bi) {
    const KeyBlock blk = s_blk[bi];
    __syncthreads();
    stage_rows<kHKB>(sK, (blk.slot < 0 ? LK : GK) + blk.row0 * 64, blk.rows, tid);
    __syncthreads();
    float s0, s1;
    bool ok0, ok1;
    score(blk, 0, s0, ok0);
    score(blk, 1, s1, ok1);
    float bm = fmaxf(ok0 ? s0 : -INFINITY, ok1 ? s1 : -INFINITY);
    bm = half_warp_max(bm);
    // nm is uniform over a half warp only: every shuffle stays outside the
    // branch so that both halves of the warp take part.
    const float nm = fmaxf(m, bm);
    float add = (ok0 ? __expf(s0 - nm) : 0.f) + (ok1 ? __expf(s1 - nm) : 0.f);
    add = half_warp_sum(add);
    if (nm > -INFINITY) {
      l = (m > -INFINITY ? l * __expf(m - nm) : 0.f) + add;
      m = nm;
    }
  }
  const float lse = l > 0.f ? m + __logf(l) : INFINITY;  // +inf: no keys, P = 0
  const float delta = s_delta[qi];

  // ---- pass 2: gradients
  float dq[4] = {0.f, 0.f, 0.f, 0.f};
  const int dq_q = tid >> 4, dq_d = (tid & 15) * 4;      // dq ownership (same query as the score thread)
  const int kv_k = tid >> 3, kv_d = (tid & 7) * 8;       // dK / dV ownership
  for (int bi = 0; bi < nblk; ++bi) {
    const KeyBlock blk = s_blk[bi];
    __syncthreads();
    stage_rows<kHKB>(sK, (blk.slot < 0 ? LK : GK) + blk.row0 * 64, blk.rows, tid);
    stage_rows<kHKB>(sV, (blk.slot < 0 ? LV : GV) + blk.row0 * 64, blk.rows, tid);
    __syncthreads();
    float rsum = 0.f;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float s;
      bool ok;
      score(blk, e, s, ok);
      const float p = ok ? __expf(s - lse) : 0.f;
      float dp = 0.f;
#pragma unroll 16
      for (int d = 0; d < 64; ++d) dp = fmaf(sdO[qi][d], sV[kk + e][d], dp);
      const float ds = p * (dp - delta);
      sP[qi][kk + e] = p;
      sdS[qi][kk + e] = ds;
      rsum += ds;
    }
    if (blk.slot >= 0) {
      rsum = half_warp_sum(rsum);
      if ((tid & 15) == 0) s_droute[qi][blk.slot] += rsum;
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < kHKB; ++k) {
      const float ds = sdS[dq_q][k];
#pragma unroll
      for (int i = 0; i < 4; ++i) dq[i] = fmaf(ds, sK[k][dq_d + i], dq[i]);
    }
    if (kv_k < blk.rows) {
      float dk[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, dv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      bool any = false;
#pragma unroll
      for (int q = 0; q < kHQ; ++q) {
        const float ds = sdS[q][kv_k], p = sP[q][kv_k];
        any |= p != 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          dk[i] = fmaf(ds, sQ[q][kv_d + i], dk[i]);
          dv[i] = fmaf(p, sdO[q][kv_d + i], dv[i]);
        }
      }
      if (any) {
        const int64_t row = bh + blk.row0 + kv_k;
        float* gk = (blk.slot < 0 ? a.d_local_key : a.d_global_key) + row * 64 + kv_d;
        float* gv = (blk.slot < 0 ? a.d_local_value : a.d_global_value) + row * 64 + kv_d;
        atomicAdd(reinterpret_cast<float4*>(gk), make_float4(dk[0] * kHScale, dk[1] * kHScale, dk[2] * kHScale, dk[3] * kHScale));
        atomicAdd(reinterpret_cast<float4*>(gk + 4), make_float4(dk[4] * kHScale, dk[5] * kHScale, dk[6] * kHScale, dk[7] * kHScale));
        atomicAdd(reinterpret_cast<float4*>(gv), make_float4(dv[0], dv[1], dv[2], dv[3]));
        atomicAdd(reinterpret_cast<float4*>(gv + 4), make_float4(dv[4], dv[5], dv[6], dv[7]));
      }
    }
  }
  __syncthreads();
  if (dq_q < nq) {
    *reinterpret_cast<float4*>(a.dq + (bh + n0 + dq_q) * 64 + dq_d) =
        make_float4(dq[0] * kHScale, dq[1] * kHScale, dq[2] * kHScale, dq[3] * kHScale);
  }
  if (tid < kHQ * 4 && (tid >> 2) < nq) a.d_route[(bh + n0) * 4 + tid] = s_droute[tid >> 2][tid & 3];
}

}  // namespace
}  // namespace dwarf

using namespace dwarf;

extern "C" int dwarf_hisa_attn_bwd(const dwarf_hisa_attn_bwd_args* a, void* stream) {
  DWARF_CHECK_VERSION(a);
  if (a->B < 0 || a->H <= 0 || a->T < 0 || a->k_slots < 0 || a->k_slots > 4) return DWARF_ERR_SHAPE;
  if (a->B > 65535 || a->H > 65535) return DWARF_ERR_SHAPE;
  if (a->B == 0 || a->T == 0) return DWARF_OK;
  if (!a->query || !a->local_key || !a->local_value || !a->global_key || !a->global_value || !a->route ||
      !a->lengths || !a->out || !a->dout || !a->dq || !a->d_local_key || !a->d_local_value ||
      !a->d_global_key || !a->d_global_value || !a->d_route || (a->k_slots > 0 && !a->top_chunk_idx))
    return DWARF_ERR_NULL;
  const void* rows[] = {a->query, a->local_key, a->local_value, a->global_key, a->global_value, a->out, a->dout,
                        a->dq, a->d_local_key, a->d_local_value, a->d_global_key, a->d_global_value};
  for (const void* r : rows)
    if (!aligned16(r)) return DWARF_ERR_ALIGN;
  if (reinterpret_cast<uintptr_t>(a->route) & 7u) return DWARF_ERR_ALIGN;
  const int64_t tiles = (a->T + kHQ - 1) / kHQ;
  if (tiles > 2147483647LL) return DWARF_ERR_SHAPE;
  hisa_attn_bwd_kernel<<<dim3((unsigned)tiles, (unsigned)a->H, (unsigned)a->B), kHT, 0,
                         static_cast<cudaStream_t>(stream)>>>(*a);
  return launch_status();
}
