// DSQG QKV prep: probe projections y/z and (optionally) q6 packing of K and V
// in one pass over the qkvg projection output (rows of 64 bf16 values).
//
// Replaces the y_pre/z_pre einsums of DSQGAttentionV19.forward
// (kernels/dsqg_attention_v22.py:3231-3254). 16 threads own one row, 4
// values each; norms, probe dots and the q6 row maximum are 16-lane shuffle
// reductions. Rows are numbered q rows first, then k rows, then v rows.
#include "common.cuh"
#include "q6_format.cuh"

namespace dwarf {
namespace {

struct PrepParams {
  int64_t H, Hkv, N, rows_q, rows_k;
  int pack;
  const __nv_bfloat16 *q, *k, *v;
  int64_t sqb, sqh, sqn, skb, skh, skn, svb, svh, svn;
  const float *qp, *kp;
  float *y, *z;
  uint8_t *kc, *vc;
  uint16_t *ks, *vs;
};

__device__ __forceinline__ float sum16(float v) {
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o, 16);
  return v;
}

__global__ void __launch_bounds__(256) dsqg_prep_kernel(const PrepParams p) {
  const int64_t row = (int64_t)blockIdx.x * 16 + threadIdx.x / 16;
  const int g = threadIdx.x & 15;
  const int64_t rows_v = p.pack ? p.rows_k : 0;
  const int64_t total = p.rows_q + p.rows_k + rows_v;
  const bool active = row < total;
  int kind = 0;  // 0 = q, 1 = k, 2 = v
  int64_t r = active ? row : 0;
  if (r >= p.rows_q) { r -= p.rows_q; kind = 1; if (r >= p.rows_k) { r -= p.rows_k; kind = 2; } }
  const int64_t heads = kind == 0 ? p.H : p.Hkv;
  const int64_t t = r % p.N;
  const int64_t h = (r / p.N) % heads;
  const int64_t b = r / (p.N * heads);
  const __nv_bfloat16* src = kind == 0 ? p.q + b * p.sqb + h * p.sqh + t * p.sqn
                           : kind == 1 ? p.k + b * p.skb + h * p.skh + t * p.skn
                                       : p.v + b * p.svb + h * p.svh + t * p.svn;
  float x[4];
  {
    const uint2 w = *reinterpret_cast<const uint2*>(src + g * 4);
    x[0] = __uint_as_float(w.x << 16); x[1] = __uint_as_float(w.x & 0xffff0000u);
    x[2] = __uint_as_float(w.y << 16); x[3] = __uint_as_float(w.y & 0xffff0000u);
  }
  // Every lane runs every shuffle (the two rows of a warp may be of different
  // kinds); results are used only where they apply.
  {
    const float* probe = kind == 0 ? p.qp : p.kp;
    float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
    float dots[4];
#pragma unroll
    for (int pl = 0; pl < 4; ++pl) {
      const float* pr = probe + pl * 64 + g * 4;
      dots[pl] = x[0] * pr[0] + x[1] * pr[1] + x[2] * pr[2] + x[3] * pr[3];
    }
    ss = sum16(ss);
#pragma unroll
    for (int pl = 0; pl < 4; ++pl) dots[pl] = sum16(dots[pl]);
    const float inv = rsqrtf(ss + 1e-6f * 64.0f);
    if (active && kind < 2 && g < 4) {
      float* dst = (kind == 0 ? p.y : p.z) + ((b * heads + h) * p.N + t) * 4;
      const float dg = g == 0 ? dots[0] : g == 1 ? dots[1] : g == 2 ? dots[2] : dots[3];
      dst[g] = dg * inv;
    }
  }
  if (p.pack) {
    float amax = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
#pragma unroll
    for (int o = 8; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o, 16));
    const __half s = q6_scale_from_amax(amax);
    const float sf = __half2float(s);
    uint32_t w = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) w |= (uint32_t)(q6_quantize(x[i], sf) & 63) << (6 * i);
    if (active && kind > 0) {
      const int64_t rr = (b * p.Hkv + h) * p.N + t;
      uint8_t* dst = (kind == 1 ? p.kc : p.vc) + rr * 48 + g * 3;
      dst[0] = (uint8_t)(w & 255u);
      dst[1] = (uint8_t)((w >> 8) & 255u);
      dst[2] = (uint8_t)((w >> 16) & 255u);
      if (g == 0) (kind == 1 ? p.ks : p.vs)[rr] = __half_as_ushort(s);
    }
  }
}

}  // namespace
}  // namespace dwarf

using namespace dwarf;

extern "C" int dwarf_dsqg_prep(const dwarf_dsqg_prep_args* a, void* stream) {
  DWARF_CHECK_VERSION(a);
  if (a->B < 0 || a->H <= 0 || a->H_kv <= 0 || a->N < 0 || a->H % a->H_kv) return DWARF_ERR_SHAPE;
  if (a->B == 0 || a->N == 0) return DWARF_OK;
  if (!a->q || !a->k || !a->q_probe || !a->k_probe || !a->y_pre || !a->z_pre) return DWARF_ERR_NULL;
  if (a->pack_q6 && (!a->v || !a->k_codes || !a->k_scales || !a->v_codes || !a->v_scales)) return DWARF_ERR_NULL;
  auto al8 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 7u) == 0; };
  if (!al8(a->q) || !al8(a->k) || (a->pack_q6 && !al8(a->v))) return DWARF_ERR_ALIGN;
  if ((a->sqb | a->sqh | a->sqn | a->skb | a->skh | a->skn) % 4 != 0) return DWARF_ERR_ALIGN;
  if (a->pack_q6 && (a->svb | a->svh | a->svn) % 4 != 0) return DWARF_ERR_ALIGN;
  PrepParams p{};
  p.H = a->H; p.Hkv = a->H_kv; p.N = a->N;
  p.rows_q = a->B * a->H * a->N;
  p.rows_k = a->B * a->H_kv * a->N;
  p.pack = a->pack_q6 ? 1 : 0;
  p.q = (const __nv_bfloat16*)a->q; p.k = (const __nv_bfloat16*)a->k; p.v = (const __nv_bfloat16*)a->v;
  p.sqb = a->sqb; p.sqh = a->sqh; p.sqn = a->sqn;
  p.skb = a->skb; p.skh = a->skh; p.skn = a->skn;
  p.svb = a->svb; p.svh = a->svh; p.svn = a->svn;
  p.qp = a->q_probe; p.kp = a->k_probe; p.y = a->y_pre; p.z = a->z_pre;
  p.kc = a->k_codes; p.vc = a->v_codes; p.ks = a->k_scales; p.vs = a->v_scales;
  const int64_t total = p.rows_q + p.rows_k + (p.pack ? p.rows_k : 0);
  const int64_t blocks = (total + 15) / 16;
  if (blocks > 0x7fffffffLL) return DWARF_ERR_SHAPE;
  dsqg_prep_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(p);
  return launch_status();
}
