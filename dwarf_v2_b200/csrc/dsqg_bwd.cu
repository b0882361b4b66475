// DSQG lattice attention backward over bf16 K/V: the gradients of
// _DSQGV18GroupedFn (kernels/dsqg_attention_v22.py:2354-2552; its Triton
// kernels _compute_D_v18_grouped, _bwd_dq_v18_grouped, _bwd_dkdv_v18_grouped
// :1263-2196), restated as two gather kernels:
//
// * query side: one query row per 4 threads (16 head dims each; thread t owns
//   MOVT plane t, whose channel pair 16 t + shift, + 1 lies in its 16 dims).
//   Recomputes each pair's probability from the forward's lse, then dq,
//   dy_pre, delta = dO . O, the per-pair ds (for the caller's pos_bias /
//   scale_embed reductions) and the phase-table gradients (summed over the
//   warp's 8 queries with shuffles, over the CTA in shared memory, then one
//   global atomic per table entry and CTA);
// * key side: one source row per 4 threads, gathering the queries
//   s + off_j of every query head that reads this KV head: dk, dv, dz_pre.
//   Each output row has exactly one writer, so dk/dv need no atomics.
//
// Pairs whose offset reaches before token 0 (query side) or past the last
// token (key side) for all 8 rows of a warp are skipped warp-uniformly.
#include "common.cuh"

namespace dwarf {
namespace {

constexpr int kBThreads = 128;
constexpr int kBRows = kBThreads / 4;  // rows per CTA
constexpr int kBMaxJ = 96;
constexpr float kBScale = 0.125f;      // 1 / sqrt(64)
constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ void load16(const __nv_bfloat16* p, float (&o)[16]) {
  const uint4* s = reinterpret_cast<const uint4*>(p);
  const uint4 w[2] = {s[0], s[1]};
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint32_t u[4] = {w[i].x, w[i].y, w[i].z, w[i].w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      o[8 * i + 2 * k] = __uint_as_float(u[k] << 16);
      o[8 * i + 2 * k + 1] = __uint_as_float(u[k] & 0xffff0000u);
    }
  }
}

__device__ __forceinline__ void store16(__nv_bfloat16* p, const float (&v)[16]) {
  uint4 w[2];
  uint32_t* u = reinterpret_cast<uint32_t*>(w);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const __nv_bfloat162 two = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    u[i] = *reinterpret_cast<const uint32_t*>(&two);
  }
  uint4* d = reinterpret_cast<uint4*>(p);
  d[0] = w[0];
  d[1] = w[1];
}

// Sum over the 4 threads of a row (same value in all four).
__device__ __forceinline__ float quad_sum(float x) {
  x += __shfl_xor_sync(kFull, x, 1);
  return x + __shfl_xor_sync(kFull, x, 2);
}
// Sum over the warp's 8 rows for one quarter (lanes t, t + 4, ..., t + 28).
__device__ __forceinline__ float octet_sum(float x) {
  x += __shfl_xor_sync(kFull, x, 4);
  x += __shfl_xor_sync(kFull, x, 8);
  return x + __shfl_xor_sync(kFull, x, 16);
}
// v[i] for a runtime i in [0, 16) without local-memory indexing.
__device__ __forceinline__ float pick16(const float (&v)[16], int i) {
  float r = v[0];
#pragma unroll
  for (int k = 1; k < 16; ++k) r = i == k ? v[k] : r;
  return r;
}

struct BwdTables {
  float se[kBMaxJ][64];  // bf16-rounded scale_embed (as the forward uses it)
  float pb[kBMaxJ];
  int off[kBMaxJ];
  float pbase[kBMaxJ][4], pgain[kBMaxJ][4];
};

__device__ void load_head_tables(BwdTables& T, const dwarf_dsqg_bwd_args& a, int64_t h, int tid) {
  for (int j = tid; j < a.J; j += kBThreads) {
    T.pb[j] = a.pos_bias[j * a.H + h];
    T.off[j] = a.offsets[j];
  }
  for (int i = tid; i < a.j_large * 4; i += kBThreads) {
    const int j = i >> 2, r = i & 3;
    T.pbase[j][r] = a.phase_base[(j * a.H + h) * 4 + r];
    T.pgain[j][r] = a.phase_gain[(j * a.H + h) * 4 + r];
  }
}

__global__ void __launch_bounds__(kBThreads) dsqg_bwd_query_kernel(const dwarf_dsqg_bwd_args a) {
  __shared__ BwdTables T;
  __shared__ float s_dpbase[kBMaxJ][4], s_dpgain[kBMaxJ][4];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, t = lane & 3;
  const int64_t h = blockIdx.y, b = blockIdx.z;
  const int64_t hk = h / (a.H / a.H_kv);
  const int64_t N = a.N;
  const int J = a.J, js = a.j_small, jl_n = a.j_large;
  for (int i = tid; i < J * 64; i += kBThreads) T.se[i >> 6][i & 63] = round_bf16(a.scale_embed[i]);
  load_head_tables(T, a, h, tid);
  for (int i = tid; i < jl_n * 4; i += kBThreads) {
    s_dpbase[i >> 2][i & 3] = 0.0f;
    s_dpgain[i >> 2][i & 3] = 0.0f;
  }
  __syncthreads();

  const int64_t n = (int64_t)blockIdx.x * kBRows + (tid >> 2);
  const int64_t warp_last = (int64_t)blockIdx.x * kBRows + warp * 8 + 7;
  const bool valid_q = n < N && n >= a.query_start;
  const int64_t nn = n < N ? n : N - 1;
  const int64_t qrow = (b * a.H + h) * N + nn;
  const int64_t kvbase = (b * a.H_kv + hk) * N;
  const __nv_bfloat16* Q = static_cast<const __nv_bfloat16*>(a.q);
  const __nv_bfloat16* K = static_cast<const __nv_bfloat16*>(a.k);
  const __nv_bfloat16* V = static_cast<const __nv_bfloat16*>(a.v);
  float q[16], dO[16], o[16], dq[16];
  load16(Q + qrow * 64 + 16 * t, q);
  load16(static_cast<const __nv_bfloat16*>(a.dout) + qrow * 64 + 16 * t, dO);
  load16(static_cast<const __nv_bfloat16*>(a.out) + qrow * 64 + 16 * t, o);
  float dsum = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) { dsum = fmaf(dO[i], o[i], dsum); dq[i] = 0.0f; }
  const float delta = quad_sum(dsum);
  const float lse = valid_q ? a.lse[qrow] : 0.0f;
  const float y_t = a.y_pre[qrow * 4 + t];
  const int la = a.plane_shift, lb = a.plane_shift + 1;
  const float dOa = pick16(dO, la), dOb = pick16(dO, lb);
  float dy = 0.0f;

#pragma unroll 1
  for (int j = 0; j < J; ++j) {
    const int off = T.off[j];
    if (off > warp_last) continue;  // warp-uniform
    const int64_t s = n - off;
    const bool ok = valid_q && s >= 0;
    const int64_t src = ok ? s : 0;
    float k[16], v[16];
    load16(K + (kvbase + src) * 64 + 16 * t, k);
    load16(V + (kvbase + src) * 64 + 16 * t, v);
    float part = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      k[i] += T.se[j][16 * t + i];
      part = fmaf(q[i], k[i], part);
    }
    const float score = fmaf(quad_sum(part), kBScale, T.pb[j]);
    const float p = ok ? __expf(score - lse) : 0.0f;
    float dpart = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) dpart = fmaf(dO[i], v[i], dpart);
    const bool large = j >= js;  // warp-uniform
    float dth = 0.0f, zt = 0.0f, gain = 0.0f;
    float ra = 0.0f, rb = 0.0f;
    if (large) {
      const int jl = j - js;
      zt = a.z_pre[(kvbase + src) * 4 + t];
      gain = T.pgain[jl][t];
      const float theta = fmaf(gain * y_t, zt, T.pbase[jl][t]);
      float sn, cs;
      __sincosf(theta, &sn, &cs);
      const float va = pick16(v, la), vb = pick16(v, lb);
      ra = cs * va - sn * vb;
      rb = sn * va + cs * vb;
      dpart += dOa * (ra - va) + dOb * (rb - vb);
    }
    const float ds = p * (quad_sum(dpart) - delta);
#pragma unroll
    for (int i = 0; i < 16; ++i) dq[i] = fmaf(ds, k[i], dq[i]);
    if (t == 0 && ok) a.ds[((b * a.H + h) * N + n) * J + j] = ds;
    if (large) {
      const int jl = j - js;
      dth = p * (dOb * ra - dOa * rb);
      dy = fmaf(dth * gain, zt, dy);
      const float gb = octet_sum(dth);
      const float gg = octet_sum(dth * y_t * zt);
      if (lane < 4) {
        atomicAdd(&s_dpbase[jl][t], gb);
        atomicAdd(&s_dpgain[jl][t], gg);
      }
    }
  }
  if (n < N) {
#pragma unroll
    for (int i = 0; i < 16; ++i) dq[i] *= kBScale;
    store16(static_cast<__nv_bfloat16*>(a.dq) + ((b * a.H + h) * N + n) * 64 + 16 * t, dq);
    a.dy_pre[((b * a.H + h) * N + n) * 4 + t] = dy;
    if (t == 0) a.delta[(b * a.H + h) * N + n] = delta;
  }
  __syncthreads();
  for (int i = tid; i < jl_n * 4; i += kBThreads) {
    const int j = i >> 2, r = i & 3;
    atomicAdd(&a.d_phase_base[(j * a.H + h) * 4 + r], s_dpbase[j][r]);
    atomicAdd(&a.d_phase_gain[(j * a.H + h) * 4 + r], s_dpgain[j][r]);
  }
}

__global__ void __launch_bounds__(kBThreads) dsqg_bwd_key_kernel(const dwarf_dsqg_bwd_args a) {
  __shared__ BwdTables T;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, t = lane & 3;
  const int64_t hk = blockIdx.y, b = blockIdx.z;
  const int64_t group = a.H / a.H_kv;
  const int64_t N = a.N;
  const int J = a.J, js = a.j_small;
  for (int i = tid; i < J * 64; i += kBThreads) T.se[i >> 6][i & 63] = round_bf16(a.scale_embed[i]);

  const int64_t s = (int64_t)blockIdx.x * kBRows + (tid >> 2);
  const int64_t warp_first = (int64_t)blockIdx.x * kBRows + warp * 8;
  const bool valid_s = s < N;
  const int64_t ss = valid_s ? s : N - 1;
  const int64_t krow = (b * a.H_kv + hk) * N + ss;
  float k[16], v[16], dk[16], dv[16];
  load16(static_cast<const __nv_bfloat16*>(a.k) + krow * 64 + 16 * t, k);
  load16(static_cast<const __nv_bfloat16*>(a.v) + krow * 64 + 16 * t, v);
#pragma unroll
  for (int i = 0; i < 16; ++i) { dk[i] = 0.0f; dv[i] = 0.0f; }
  const float zt = a.z_pre[krow * 4 + t];
  const int la = a.plane_shift, lb = a.plane_shift + 1;
  const float va = pick16(v, la), vb = pick16(v, lb);
  float corr_a = 0.0f, corr_b = 0.0f, dz = 0.0f;
  const __nv_bfloat16* Q = static_cast<const __nv_bfloat16*>(a.q);
  const __nv_bfloat16* DO = static_cast<const __nv_bfloat16*>(a.dout);

#pragma unroll 1
  for (int64_t g = 0; g < group; ++g) {
    const int64_t h = hk * group + g;
    __syncthreads();  // previous head's tables are no longer read
    load_head_tables(T, a, h, tid);
    __syncthreads();
    const int64_t qbase = (b * a.H + h) * N;
#pragma unroll 1
    for (int j = 0; j < J; ++j) {
      const int off = T.off[j];
      if (warp_first + off >= N) continue;  // warp-uniform
      const int64_t n = s + off;
      const bool ok = valid_s && n < N && n >= a.query_start;
      const int64_t nq = ok ? n : 0;
      float q[16], dO[16];
      load16(Q + (qbase + nq) * 64 + 16 * t, q);
      load16(DO + (qbase + nq) * 64 + 16 * t, dO);
      const float lse = ok ? a.lse[qbase + nq] : 0.0f;
      const float delta = ok ? a.delta[qbase + nq] : 0.0f;
      float part = 0.0f, dpart = 0.0f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        part = fmaf(q[i], k[i] + T.se[j][16 * t + i], part);
        dpart = fmaf(dO[i], v[i], dpart);
      }
      const float score = fmaf(quad_sum(part), kBScale, T.pb[j]);
      const float p = ok ? __expf(score - lse) : 0.0f;
      const bool large = j >= js;  // warp-uniform
      float cs = 1.0f, sn = 0.0f, ra = va, rb = vb, yt = 0.0f, gain = 0.0f;
      if (large) {
        const int jl = j - js;
        yt = a.y_pre[(qbase + nq) * 4 + t];
        gain = T.pgain[jl][t];
        const float theta = fmaf(gain * yt, zt, T.pbase[jl][t]);
        __sincosf(theta, &sn, &cs);
        ra = cs * va - sn * vb;
        rb = sn * va + cs * vb;
      }
      const float dOa = pick16(dO, la), dOb = pick16(dO, lb);
      dpart += dOa * (ra - va) + dOb * (rb - vb);
      const float ds = p * (quad_sum(dpart) - delta);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        dk[i] = fmaf(ds, q[i], dk[i]);
        dv[i] = fmaf(p, dO[i], dv[i]);
      }
      if (large) {
        corr_a = fmaf(p, (cs - 1.0f) * dOa + sn * dOb, corr_a);
        corr_b = fmaf(p, (cs - 1.0f) * dOb - sn * dOa, corr_b);
        dz = fmaf(p * (dOb * ra - dOa * rb) * gain, yt, dz);
      }
    }
  }
  if (!valid_s) return;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    dk[i] *= kBScale;
    dv[i] += i == la ? corr_a : (i == lb ? corr_b : 0.0f);
  }
  const int64_t orow = (b * a.H_kv + hk) * N + s;
  store16(static_cast<__nv_bfloat16*>(a.dk) + orow * 64 + 16 * t, dk);
  store16(static_cast<__nv_bfloat16*>(a.dv) + orow * 64 + 16 * t, dv);
  a.dz_pre[orow * 4 + t] = dz;
}

}  // namespace
}  // namespace dwarf

using namespace dwarf;

extern "C" int dwarf_dsqg_bwd(const dwarf_dsqg_bwd_args* a, void* stream_) {
  DWARF_CHECK_VERSION(a);
  if (a->B < 0 || a->H <= 0 || a->H_kv <= 0 || a->N < 0 || a->H % a->H_kv) return DWARF_ERR_SHAPE;
  if (a->J <= 0 || a->J > kBMaxJ || a->j_small < 0 || a->j_large < 0 || a->j_small + a->j_large != a->J)
    return DWARF_ERR_SHAPE;
  if (a->plane_shift < 0 || a->plane_shift > 14 || a->query_start < 0) return DWARF_ERR_VALUE;
  if (a->B > 65535 || a->H > 65535) return DWARF_ERR_SHAPE;
  if (!a->q || !a->k || !a->v || !a->out || !a->dout || !a->lse || !a->offsets || !a->pos_bias ||
      !a->scale_embed || !a->y_pre || !a->z_pre || !a->dq || !a->dk || !a->dv || !a->dy_pre || !a->dz_pre ||
      !a->ds || !a->delta)
    return DWARF_ERR_NULL;
  if (a->j_large > 0 && (!a->phase_base || !a->phase_gain || !a->d_phase_base || !a->d_phase_gain))
    return DWARF_ERR_NULL;
  const void* rows[] = {a->q, a->k, a->v, a->out, a->dout, a->dq, a->dk, a->dv, a->y_pre, a->z_pre,
                        a->dy_pre, a->dz_pre};
  for (const void* r : rows)
    if (!aligned16(r)) return DWARF_ERR_ALIGN;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (a->j_large > 0) {
    const size_t bytes = (size_t)a->j_large * a->H * 4 * sizeof(float);
    if (cudaMemsetAsync(a->d_phase_base, 0, bytes, stream) != cudaSuccess ||
        cudaMemsetAsync(a->d_phase_gain, 0, bytes, stream) != cudaSuccess)
      return DWARF_ERR_LAUNCH;
  }
  if (a->B == 0 || a->N == 0) return DWARF_OK;
  const int64_t tiles = (a->N + kBRows - 1) / kBRows;
  if (tiles > 2147483647LL) return DWARF_ERR_SHAPE;
  dsqg_bwd_query_kernel<<<dim3((unsigned)tiles, (unsigned)a->H, (unsigned)a->B), kBThreads, 0, stream>>>(*a);
  int rc = launch_status();
  if (rc != DWARF_OK) return rc;
  dsqg_bwd_key_kernel<<<dim3((unsigned)tiles, (unsigned)a->H_kv, (unsigned)a->B), kBThreads, 0, stream>>>(*a);
  return launch_status();
}
