// DSQG lattice attention forward (CUDA cores, fp32 math).
//
// Replaces _fwd_v22_online (kernels/dsqg_attention_v22.py:698-860), launched
// by _DSQGV18GroupedFn.forward (:2197-2352). Same semantics, same order of
// offsets, same online softmax in the exp2 domain and the same bf16 rounding
// of the scale-embedding "virtual key" (:760-763); differences to the
// reference are fp32 summation order only.
//
// Mapping: one CTA = 64 consecutive queries of one (batch, head); 4 threads
// per query, each owning 16 of the 64 head dims (32 B of a bf16 row, or 12 B
// of a q6 row). A query's dot product is reduced over its 4 threads with two
// xor-shuffles. MOVT plane r (channels 16r+shift, 16r+shift+1) lies inside the
// slice of thread r, so each thread rotates exactly one plane. K/V rows are
// gathered straight from global memory (rows of neighbouring queries are
// neighbouring rows, so each warp reads 8 whole rows per offset), with the
// next offset's rows prefetched while the current one is consumed.
// Per-offset tables (offsets, pos_bias[:,h], bf16(scale_embed), this head's
// phase base/gain) are staged in shared memory once per CTA.
#include "common.cuh"
#include "q6_format.cuh"

namespace dwarf {
namespace {

constexpr int kQB = 64;       // queries per CTA
constexpr int kThreads = 256;  // 4 per query
constexpr float kLog2e = 1.4426950408889634f;

struct DsqgParams {
  int64_t H, Hkv, N;
  int J, j_small, j_large, plane_shift, query_start, kv_group;
  const __nv_bfloat16* q;
  int64_t sqb, sqh, sqn;
  const __nv_bfloat16* k;
  int64_t skb, skh, skn;
  const __nv_bfloat16* v;
  int64_t svb, svh, svn;
  const uint8_t* kc;
  const uint16_t* ks;
  const uint8_t* vc;
  const uint16_t* vs;
  int64_t ccb, cch, cct, csb, csh, cst;
  const int32_t* offsets;
  const float* pos_bias;
  int64_t spj, sph;
  const float* se;
  int64_t sej, sed;
  const float* pbase;
  int64_t sbj, sbh;
  const float* pgain;
  int64_t sgj, sgh;
  const float* y;
  int64_t syb, syh, syn;
  const float* z;
  int64_t szb, szh, szn;
  __nv_bfloat16* out;
  int64_t sob, soh, son;
  float* lse;
  int64_t slb, slh, sln;
  const void* gain;
  int gain_bf16;
  const __nv_bfloat16* gate;
  int64_t sgtb, sgtn;
};

// 16 bf16 (two 16-B words) -> 16 floats.
__device__ __forceinline__ void bf16x16_to_f32(const uint4 (&w)[2], float (&o)[16]) {
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint32_t u[4] = {w[i].x, w[i].y, w[i].z, w[i].w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      o[i * 8 + 2 * k] = __uint_as_float(u[k] << 16);
      o[i * 8 + 2 * k + 1] = __uint_as_float(u[k] & 0xffff0000u);
    }
  }
}

template <int I>
__device__ __forceinline__ void q6_decode16_impl(const uint32_t (&w)[3], float step, float (&o)[16]) {
  if constexpr (I < 16) {
    o[I] = (float)q6_code96<I>(w) * step;
    q6_decode16_impl<I + 1>(w, step, o);
  }
}

// One gathered row slice: bf16 (2 x uint4) or q6 (3 x u32 + fp16 scale).
template <bool Q6>
struct RowSlice;
template <>
struct RowSlice<false> {
  uint4 w[2];
  __device__ __forceinline__ void load(const __nv_bfloat16* base, bool ok) {
    if (ok) {
      const uint4* p = reinterpret_cast<const uint4*>(base);
      w[0] = __ldg(p);
      w[1] = __ldg(p + 1);
    } else {
      w[0] = w[1] = make_uint4(0, 0, 0, 0);
    }
  }
  __device__ __forceinline__ void to_f32(float (&o)[16]) const { bf16x16_to_f32(w, o); }
};
template <>
struct RowSlice<true> {
  uint32_t w[3];
  uint16_t s;
  __device__ __forceinline__ void load(const uint8_t* codes, const uint16_t* scale, bool ok) {
    if (ok) {
      const uint32_t* p = reinterpret_cast<const uint32_t*>(codes);
      w[0] = __ldg(p);
      w[1] = __ldg(p + 1);
      w[2] = __ldg(p + 2);
      s = __ldg(scale);
    } else {
      w[0] = w[1] = w[2] = 0u;
      s = 0;
    }
  }
  __device__ __forceinline__ void to_f32(float (&o)[16]) const {
    q6_decode16_impl<0>(w, q6_step(__ushort_as_half(s)), o);
  }
};

template <bool Q6>
__global__ void __launch_bounds__(kThreads)
dsqg_fwd_kernel(const DsqgParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int J = p.J;
  float* s_se = reinterpret_cast<float*>(smem);            // [J][64]
  float* s_pb = s_se + (size_t)J * 64;                     // [J]
  int* s_off = reinterpret_cast<int*>(s_pb + J);           // [J]
  float* s_pbase = reinterpret_cast<float*>(s_off + J);    // [j_large][4]
  float* s_pgain = s_pbase + (size_t)p.j_large * 4;        // [j_large][4]
  __shared__ int s_count[2];

  const int64_t b = blockIdx.z;
  const int64_t h = blockIdx.y;
  const int64_t hk = h / p.kv_group;
  const int sub = threadIdx.x & 3;
  const int64_t n = (int64_t)blockIdx.x * kQB + (threadIdx.x >> 2);
  const int64_t n_end = (int64_t)blockIdx.x * kQB + kQB;
  const int64_t n_last = (n_end < p.N ? n_end : p.N) - 1;

  for (int i = threadIdx.x; i < J * 64; i += kThreads) {
    const int j = i >> 6, d = i & 63;
    s_se[i] = round_bf16(p.se[j * p.sej + d * p.sed]);
  }
  for (int j = threadIdx.x; j < J; j += kThreads) {
    s_pb[j] = p.pos_bias[j * p.spj + h * p.sph];
    s_off[j] = p.offsets[j];
  }
  for (int i = threadIdx.x; i < p.j_large * 4; i += kThreads) {
    const int j = i >> 2, r = i & 3;
    s_pbase[i] = p.pbase[j * p.sbj + h * p.sbh + r];
    s_pgain[i] = p.pgain[j * p.sgj + h * p.sgh + r];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // Offsets are ascending inside each band: the ones this CTA can use are a
    // prefix of the small band and a prefix of the large band.
    int cs = 0, cl = 0;
    for (int j = 0; j < p.j_small; ++j) cs += (s_off[j] <= n_last);
    for (int j = p.j_small; j < J; ++j) cl += (s_off[j] <= n_last);
    s_count[0] = cs;
    s_count[1] = cl;
  }
  __syncthreads();
  const int count_small = s_count[0];
  const int count_large = s_count[1];
  const int steps = count_small + count_large;

  const bool row_ok = n < p.N && n >= p.query_start;
  const int64_t nn = n < p.N ? n : p.N - 1;
  const int d0 = sub * 16;

  float q[16];
  {
    RowSlice<false> qs;
    qs.load(p.q + b * p.sqb + h * p.sqh + nn * p.sqn + d0, true);
    qs.to_f32(q);
  }
  const float yq = p.y[b * p.syb + h * p.syh + nn * p.syn + sub];
  const int rot_a = p.plane_shift;  // local channel of this thread's plane

  float acc[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i] = 0.0f;
  float m = -INFINITY, l = 0.0f;

  auto jof = [&](int step) { return step < count_small ? step : p.j_small + (step - count_small); };

  RowSlice<Q6> kn, vn;
  float zn = 0.0f;
  auto fetch = [&](int step, RowSlice<Q6>& kr, RowSlice<Q6>& vr, float& zr) {
    const int j = jof(step);
    const int64_t src = n - s_off[j];
    const bool ok = row_ok && src >= 0;
    const int64_t s = ok ? src : 0;
    if constexpr (Q6) {
      kr.load(p.kc + b * p.ccb + hk * p.cch + s * p.cct + sub * 12, p.ks + b * p.csb + hk * p.csh + s * p.cst, ok);
      vr.load(p.vc + b * p.ccb + hk * p.cch + s * p.cct + sub * 12, p.vs + b * p.csb + hk * p.csh + s * p.cst, ok);
    } else {
      kr.load(p.k + b * p.skb + hk * p.skh + s * p.skn + d0, ok);
      vr.load(p.v + b * p.svb + hk * p.svh + s * p.svn + d0, ok);
    }
    zr = (ok && j >= p.j_small) ? __ldg(p.z + b * p.szb + hk * p.szh + s * p.szn + sub) : 0.0f;
  };
  if (steps > 0) fetch(0, kn, vn, zn);

  for (int step = 0; step < steps; ++step) {
    const RowSlice<Q6> kc = kn, vc = vn;
    const float zc = zn;
    if (step + 1 < steps) fetch(step + 1, kn, vn, zn);
    const int j = jof(step);
    const bool valid = row_ok && n - s_off[j] >= 0;

    float kv[16];
    kc.to_f32(kv);
    const float* e = s_se + j * 64 + d0;
    float part = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) part = fmaf(q[i], kv[i] + e[i], part);
    part += __shfl_xor_sync(0xffffffffu, part, 1);
    part += __shfl_xor_sync(0xffffffffu, part, 2);
    if (!valid) continue;  // uniform across the 4 threads of a query
    const float score = part * 0.125f + s_pb[j];

    const float m_new = fmaxf(m, score);
    const float old_scale = l > 0.0f ? exp2f((m - m_new) * kLog2e) : 0.0f;
    const float w = exp2f((score - m_new) * kLog2e);
    vc.to_f32(kv);
    if (j >= p.j_small) {
      const int jl = j - p.j_small;
      const float theta = s_pbase[jl * 4 + sub] + s_pgain[jl * 4 + sub] * yq * zc;
      float sn, cs;
      sincosf(theta, &sn, &cs);
#pragma unroll
      for (int i = 0; i < 15; ++i) {
        if (i == rot_a) {
          const float va = kv[i], vb = kv[i + 1];
          kv[i] = cs * va - sn * vb;
          kv[i + 1] = sn * va + cs * vb;
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = fmaf(acc[i], old_scale, w * kv[i]);
    l = l * old_scale + w;
    m = m_new;
  }

  if (n >= p.N) return;
  const float inv = 1.0f;
  (void)inv;
  float o[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i] = l > 0.0f ? round_bf16(acc[i] / l) : 0.0f;
  if (p.gain != nullptr) {
    const float g = p.gain_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.gain)[h])
                                : reinterpret_cast<const float*>(p.gain)[h];
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i] = p.gain_bf16 ? round_bf16(o[i] * g) : o[i] * g;
  }
  if (p.gate != nullptr) {
    RowSlice<false> gs;
    gs.load(p.gate + b * p.sgtb + n * p.sgtn + h * 64 + d0, true);
    float gv[16];
    gs.to_f32(gv);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float sg = round_bf16(1.0f / (1.0f + expf(-gv[i])));
      o[i] = p.gain_bf16 || p.gain == nullptr ? round_bf16(o[i] * sg) : o[i] * sg;
    }
  }
  uint4 packed[2];
  uint32_t* pw = reinterpret_cast<uint32_t*>(packed);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const __nv_bfloat162 two = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
    pw[i] = *reinterpret_cast<const uint32_t*>(&two);
  }
  uint4* dst = reinterpret_cast<uint4*>(p.out + b * p.sob + h * p.soh + n * p.son + d0);
  dst[0] = packed[0];
  dst[1] = packed[1];
  if (p.lse != nullptr && sub == 0) {
    p.lse[b * p.slb + h * p.slh + n * p.sln] = l > 0.0f ? m + log2f(l) * (1.0f / kLog2e) : -INFINITY;
  }
}

bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool a4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

}  // namespace
}  // namespace dwarf

using namespace dwarf;

extern "C" int dwarf_dsqg_fwd(const dwarf_dsqg_fwd_args* a, void* stream) {
  DWARF_CHECK_VERSION(a);
  if (a->kv_format != 0 && a->kv_format != 1) return DWARF_ERR_VALUE;
  if (a->head_dim != 64) return DWARF_ERR_SHAPE;
  if (a->B < 0 || a->H <= 0 || a->H_kv <= 0 || a->N < 0 || a->H % a->H_kv != 0) return DWARF_ERR_SHAPE;
  if (a->J < 1 || a->j_small < 0 || a->j_large < 0 || a->j_small + a->j_large != a->J || a->J > 512)
    return DWARF_ERR_SHAPE;
  if (a->plane_shift < 0 || a->plane_shift > 14) return DWARF_ERR_VALUE;
  if (a->B == 0 || a->N == 0) return DWARF_OK;
  if (!a->q || !a->out || !a->offsets || !a->pos_bias || !a->scale_embed || !a->y_pre || !a->z_pre)
    return DWARF_ERR_NULL;
  if (a->j_large > 0 && (!a->phase_base || !a->phase_gain)) return DWARF_ERR_NULL;
  const bool q6 = a->kv_format == 1;
  if (q6) {
    if (!a->k_codes || !a->v_codes || !a->k_scales || !a->v_scales) return DWARF_ERR_NULL;
    if (!a4(a->k_codes) || !a4(a->v_codes) || (a->ccb | a->cch | a->cct) % 4 != 0) return DWARF_ERR_ALIGN;
  } else {
    if (!a->k || !a->v) return DWARF_ERR_NULL;
    if (!a16(a->k) || !a16(a->v) || (a->skb | a->skh | a->skn | a->svb | a->svh | a->svn) % 8 != 0)
      return DWARF_ERR_ALIGN;
  }
  if (!a16(a->q) || !a16(a->out) || (a->sqb | a->sqh | a->sqn | a->sob | a->soh | a->son) % 8 != 0)
    return DWARF_ERR_ALIGN;
  if (a->gate != nullptr && (!a16(a->gate) || (a->sgb_ | a->sgn_) % 8 != 0)) return DWARF_ERR_ALIGN;
  if (a->head_gain != nullptr && a->head_gain_dtype != DWARF_F32 && a->head_gain_dtype != DWARF_BF16)
    return DWARF_ERR_DTYPE;

  DsqgParams p{};
  p.H = a->H; p.Hkv = a->H_kv; p.N = a->N;
  p.J = a->J; p.j_small = a->j_small; p.j_large = a->j_large;
  p.plane_shift = a->plane_shift;
  p.query_start = a->query_start < 0 ? 0 : a->query_start;
  p.kv_group = (int)(a->H / a->H_kv);
  p.q = (const __nv_bfloat16*)a->q; p.sqb = a->sqb; p.sqh = a->sqh; p.sqn = a->sqn;
  p.k = (const __nv_bfloat16*)a->k; p.skb = a->skb; p.skh = a->skh; p.skn = a->skn;
  p.v = (const __nv_bfloat16*)a->v; p.svb = a->svb; p.svh = a->svh; p.svn = a->svn;
  p.kc = a->k_codes; p.ks = a->k_scales; p.vc = a->v_codes; p.vs = a->v_scales;
  p.ccb = a->ccb; p.cch = a->cch; p.cct = a->cct; p.csb = a->csb; p.csh = a->csh; p.cst = a->cst;
  p.offsets = a->offsets;
  p.pos_bias = a->pos_bias; p.spj = a->spj; p.sph = a->sph;
  p.se = a->scale_embed; p.sej = a->sej; p.sed = a->sed;
  p.pbase = a->phase_base; p.sbj = a->sbj; p.sbh = a->sbh;
  p.pgain = a->phase_gain; p.sgj = a->sgj; p.sgh = a->sgh;
  p.y = a->y_pre; p.syb = a->syb; p.syh = a->syh; p.syn = a->syn;
  p.z = a->z_pre; p.szb = a->szb; p.szh = a->szh; p.szn = a->szn;
  p.out = (__nv_bfloat16*)a->out; p.sob = a->sob; p.soh = a->soh; p.son = a->son;
  p.lse = a->lse; p.slb = a->slb; p.slh = a->slh; p.sln = a->sln;
  p.gain = a->head_gain; p.gain_bf16 = a->head_gain_dtype == DWARF_BF16;
  p.gate = (const __nv_bfloat16*)a->gate; p.sgtb = a->sgb_; p.sgtn = a->sgn_;

  const size_t smem = (size_t)a->J * 64 * 4 + (size_t)a->J * 8 + (size_t)a->j_large * 32;
  dim3 grid((unsigned)((a->N + kQB - 1) / kQB), (unsigned)a->H, (unsigned)a->B);
  if (grid.z > 65535 || grid.y > 65535) return DWARF_ERR_SHAPE;
  if (q6) {
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(dsqg_fwd_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem))
      return DWARF_ERR_LAUNCH;
    dsqg_fwd_kernel<true><<<grid, kThreads, smem, (cudaStream_t)stream>>>(p);
  } else {
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(dsqg_fwd_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem))
      return DWARF_ERR_LAUNCH;
    dsqg_fwd_kernel<false><<<grid, kThreads, smem, (cudaStream_t)stream>>>(p);
  }
  return launch_status();
}
