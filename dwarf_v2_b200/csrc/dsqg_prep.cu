// DSQG QKV prep: probe projections y/z and (optionally) q6 packing of K and V
// in one pass over the qkvg projection output (rows of 64 bf16 values).
//
// Replaces the y_pre/z_pre einsums of DSQGAttentionV19.forward
// (kernels/dsqg_attention_v22.py:3231-3254). 16 threads own one row, 4
// values each; norms, probe dots and the q6 row maximum are 16-lane shuffle
// reductions; the q6 row is assembled in shared memory and written as three
// 16-byte stores.
#include "common.cuh"
#include "q6_format.cuh"

namespace dwarf {
namespace {

struct PrepParams {
  int64_t H, Hkv, N;
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

constexpr int kRowGroups = 8;  // 16-row groups per CTA (128 rows)

// grid = (ceil(N/128), H + Hkv (+ Hkv when packing), B); blockIdx.y picks the
// tensor and head: [0, H) query heads, [H, H+Hkv) key heads, then value heads.
// 128 rows per CTA in groups of 16, 16 lanes per row, 4 values per lane.
__global__ void __launch_bounds__(256) dsqg_prep_kernel(const PrepParams p) {
  __shared__ float probes[2][4][64];
  __shared__ __align__(16) uint8_t codes[16][48];
  for (int i = threadIdx.x; i < 2 * 4 * 64; i += 256)
    probes[i / 256][(i / 64) & 3][i & 63] = (i < 256 ? p.qp : p.kp)[i & 255];
  __syncthreads();
  const int g = threadIdx.x & 15;
  const int lr = threadIdx.x >> 4;  // local row
  const int64_t b = blockIdx.z;
  int hy = blockIdx.y, kind = 0;
  if (hy >= p.H) { hy -= (int)p.H; kind = 1; if (hy >= p.Hkv) { hy -= (int)p.Hkv; kind = 2; } }
  const __nv_bfloat16* base = kind == 0 ? p.q + b * p.sqb + hy * p.sqh
                            : kind == 1 ? p.k + b * p.skb + hy * p.skh
                                        : p.v + b * p.svb + hy * p.svh;
  const int64_t srow = kind == 0 ? p.sqn : kind == 1 ? p.skn : p.svn;
  // All eight groups' loads are issued before any math, so each thread keeps
  // 64 B in flight (the loop below alone would expose one load latency per group).
  uint2 xw[kRowGroups];
#pragma unroll
  for (int grp = 0; grp < kRowGroups; ++grp) {
    const int64_t t = ((int64_t)blockIdx.x * kRowGroups + grp) * 16 + lr;
    const int64_t tt = t < p.N ? t : p.N - 1;
    xw[grp] = __ldg(reinterpret_cast<const uint2*>(base + tt * srow + g * 4));
  }
#pragma unroll
  for (int grp = 0; grp < kRowGroups; ++grp) {
    const int64_t t = ((int64_t)blockIdx.x * kRowGroups + grp) * 16 + lr;
    const bool active = t < p.N;
    float x[4];
    {
      const uint2 w = xw[grp];
      x[0] = __uint_as_float(w.x << 16); x[1] = __uint_as_float(w.x & 0xffff0000u);
      x[2] = __uint_as_float(w.y << 16); x[3] = __uint_as_float(w.y & 0xffff0000u);
    }
    const int heads = kind == 0 ? (int)p.H : (int)p.Hkv;
    // kind is uniform over the CTA, so these branches never split a warp.
    if (kind < 2) {
      const float (*pr)[64] = probes[kind];
      float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
      float dots[4];
  #pragma unroll
      for (int pl = 0; pl < 4; ++pl)
        dots[pl] = x[0] * pr[pl][g * 4] + x[1] * pr[pl][g * 4 + 1] + x[2] * pr[pl][g * 4 + 2] + x[3] * pr[pl][g * 4 + 3];
      ss = sum16(ss);
  #pragma unroll
      for (int pl = 0; pl < 4; ++pl) dots[pl] = sum16(dots[pl]);
      const float inv = rsqrtf(ss + 1e-6f * 64.0f);
      if (active && g == 0) {
        float* dst = (kind == 0 ? p.y : p.z) + ((b * heads + hy) * p.N + t) * 4;
        *reinterpret_cast<float4*>(dst) = make_float4(dots[0] * inv, dots[1] * inv, dots[2] * inv, dots[3] * inv);
      }
    }
    if (p.pack && kind > 0) {
      float amax = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
  #pragma unroll
      for (int o = 8; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o, 16));
      const __half s = q6_scale_from_amax(amax);
      const float inv = q6_inv_step(__half2float(s));
      uint32_t w = 0;
  #pragma unroll
      for (int i = 0; i < 4; ++i) w |= (uint32_t)(q6_quantize(x[i], inv) & 63) << (6 * i);
      codes[lr][g * 3] = (uint8_t)(w & 255u);
      codes[lr][g * 3 + 1] = (uint8_t)((w >> 8) & 255u);
      codes[lr][g * 3 + 2] = (uint8_t)((w >> 16) & 255u);
      __syncwarp();
      const int64_t rr = (b * p.Hkv + hy) * p.N + t;
      if (active && g < 3)
        reinterpret_cast<uint4*>((kind == 1 ? p.kc : p.vc) + rr * 48)[g] = reinterpret_cast<const uint4*>(codes[lr])[g];
      if (active && g == 3) (kind == 1 ? p.ks : p.vs)[rr] = __half_as_ushort(s);
    }
    __syncwarp();  // codes[] rows are reused by the next group
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
  p.pack = a->pack_q6 ? 1 : 0;
  p.q = (const __nv_bfloat16*)a->q; p.k = (const __nv_bfloat16*)a->k; p.v = (const __nv_bfloat16*)a->v;
  p.sqb = a->sqb; p.sqh = a->sqh; p.sqn = a->sqn;
  p.skb = a->skb; p.skh = a->skh; p.skn = a->skn;
  p.svb = a->svb; p.svh = a->svh; p.svn = a->svn;
  p.qp = a->q_probe; p.kp = a->k_probe; p.y = a->y_pre; p.z = a->z_pre;
  p.kc = a->k_codes; p.vc = a->v_codes; p.ks = a->k_scales; p.vs = a->v_scales;
  const int64_t ys = a->H + a->H_kv + (p.pack ? a->H_kv : 0);
  const int64_t rows_per_cta = 16 * kRowGroups;
  if (ys > 65535 || a->B > 65535 || (a->N + rows_per_cta - 1) / rows_per_cta > 0x7fffffffLL) return DWARF_ERR_SHAPE;
  dim3 grid((unsigned)((a->N + rows_per_cta - 1) / rows_per_cta), (unsigned)ys, (unsigned)a->B);
  dsqg_prep_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(p);
  return launch_status();
}
