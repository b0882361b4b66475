// NPCI magnitude-aware rotation: one 64-value head row per 8 threads (bf16
// rows with 16-byte aligned starts: one 16-byte access per tensor and lane) or
// per 16 threads (any other layout).
//
// Replaces npci_rotate (kernels/dsqg_attention_v22.py:223-254) and the
// identical _magnitude_aware_rotate (kernels/hierarchical_sparse_attn_v18_hisa.py:99-125),
// which run as ~15 separate elementwise/reduction passes in the reference.
// Three row reductions: |x|^2, d.u, then |p|^2 of the explicit perpendicular p = d - (d.u) u, as the reference computes it.
#include "common.cuh"

namespace dwarf {
namespace {

struct NpciParams {
  int64_t B, H, N;
  const void* x; int64_t sxb, sxh, sxn;
  const void* add; int64_t sab, sah, san;
  const void* d; int64_t sdb, sdh, sdn;
  const float* theta;
  float tau;
  void* out; int64_t sob, soh, son;
};

__device__ __forceinline__ float sum16(float v) {
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o, 16);
  return v;
}

template <typename T>
__device__ __forceinline__ void load4(const void* base, int64_t off, float (&v)[4]) {
  const T* p = static_cast<const T*>(base) + off;
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = static_cast<float>(p[i]);
}

template <typename T>
__device__ __forceinline__ void npci_row(const NpciParams& p, int64_t b, int64_t h, int64_t n, bool active_row,
                                         int g) {
  float x[4], d[4];
  load4<T>(p.x, b * p.sxb + h * p.sxh + n * p.sxn + g * 4, x);
  if (p.add != nullptr) {
    float a[4];
    load4<T>(p.add, b * p.sab + h * p.sah + n * p.san + g * 4, a);
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = static_cast<float>(static_cast<T>(x[i] + a[i]));
  }
  if (p.d != nullptr) {
    load4<T>(p.d, b * p.sdb + h * p.sdh + n * p.sdn + g * 4, d);
  } else {
    d[0] = d[1] = d[2] = d[3] = 0.0f;  // no packet: plain (adapter) add
  }
  float xx = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) xx += x[i] * x[i];
  const float norm = fmaxf(sqrtf(sum16(xx)), 1e-12f);
  const float inv_norm = 1.0f / norm;
  float u[4], du = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) { u[i] = x[i] * inv_norm; du += d[i] * u[i]; }
  du = sum16(du);
  float perp[4], pp = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) { perp[i] = d[i] - du * u[i]; pp += perp[i] * perp[i]; }
  const float pn = sqrtf(sum16(pp));
  const bool active = pn > norm * 1e-7f;
  // |angle| <= |theta| (0.25 rad in the DWARF blocks): there the SFU sine and
  // cosine are accurate to a few 1e-7 absolute; larger angles take sincosf.
  // tanh (of a non-negative argument) from the SFU exponential.
  const float z = pn / (p.tau * norm + 1e-12f);
  const float e2 = __expf(-2.0f * fminf(z, 40.0f));
  const float angle = p.theta[h] * __fdividef(1.0f - e2, 1.0f + e2);
  float sn, cs;
  if (fabsf(angle) < 1.0f) __sincosf(angle, &sn, &cs);
  else sincosf(angle, &sn, &cs);
  const float inv_pn = 1.0f / fmaxf(pn, 1e-20f);
  if (!active_row) return;
  T* o = static_cast<T*>(p.out) + b * p.sob + h * p.soh + n * p.son + g * 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float dir = active ? perp[i] * inv_pn : 0.0f;
    const float rot = cs * x[i] + sn * norm * dir;
    o[i] = static_cast<T>(active ? rot : x[i]);
  }
}

// bf16 rows with 16-byte aligned starts: 8 lanes per 64-value row, one 16-byte
// load per tensor and lane (8 values), three-round reductions.
__device__ __forceinline__ float sum8(float v) {
#pragma unroll
  for (int o = 4; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o, 8);
  return v;
}

__device__ __forceinline__ void npci_row_vec8(const NpciParams& p, int64_t b, int64_t h, int64_t n, bool active_row,
                                              int g) {
  float x[8], d[8];
  VecIO<__nv_bfloat16, 8>::load(static_cast<const __nv_bfloat16*>(p.x) + b * p.sxb + h * p.sxh + n * p.sxn + g * 8, x);
  if (p.add != nullptr) {
    float a[8];
    VecIO<__nv_bfloat16, 8>::load(static_cast<const __nv_bfloat16*>(p.add) + b * p.sab + h * p.sah + n * p.san + g * 8,
                                  a);
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = __bfloat162float(__float2bfloat16_rn(x[i] + a[i]));
  }
  if (p.d != nullptr) {
    VecIO<__nv_bfloat16, 8>::load(static_cast<const __nv_bfloat16*>(p.d) + b * p.sdb + h * p.sdh + n * p.sdn + g * 8, d);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) d[i] = 0.0f;
  }
  float xx = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) xx += x[i] * x[i];
  const float norm = fmaxf(sqrtf(sum8(xx)), 1e-12f);
  const float inv_norm = 1.0f / norm;
  float u[8], du = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) { u[i] = x[i] * inv_norm; du += d[i] * u[i]; }
  du = sum8(du);
  float perp[8], pp = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) { perp[i] = d[i] - du * u[i]; pp += perp[i] * perp[i]; }
  const float pn = sqrtf(sum8(pp));
  const bool active = pn > norm * 1e-7f;
  const float z = pn / (p.tau * norm + 1e-12f);
  const float e2 = __expf(-2.0f * fminf(z, 40.0f));
  const float angle = p.theta[h] * __fdividef(1.0f - e2, 1.0f + e2);
  float sn, cs;
  if (fabsf(angle) < 1.0f) __sincosf(angle, &sn, &cs);
  else sincosf(angle, &sn, &cs);
  const float inv_pn = 1.0f / fmaxf(pn, 1e-20f);
  if (!active_row) return;
  float o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float dir = active ? perp[i] * inv_pn : 0.0f;
    o[i] = active ? cs * x[i] + sn * norm * dir : x[i];
  }
  VecIO<__nv_bfloat16, 8>::store(static_cast<__nv_bfloat16*>(p.out) + b * p.sob + h * p.soh + n * p.son + g * 8, o);
}

constexpr int kRowGroups = 8;  // 16-row groups per CTA

// grid = (ceil(N / 256), H, B): 32 rows per pass of 256 threads (8 lanes per row), 8 passes.
__global__ void __launch_bounds__(256) npci_vec8_kernel(const NpciParams p) {
  const int64_t h = blockIdx.y, b = blockIdx.z;
  const int g = threadIdx.x & 7;
  for (int grp = 0; grp < kRowGroups; ++grp) {
    const int64_t row = ((int64_t)blockIdx.x * kRowGroups + grp) * 32 + threadIdx.x / 8;
    npci_row_vec8(p, b, h, row < p.N ? row : p.N - 1, row < p.N, g);
  }
}

// grid = (ceil(N / 128), H, B): each CTA rotates 128 consecutive tokens of one
// (b, h), 16 lanes per 64-value row.
template <typename T>
__global__ void __launch_bounds__(256) npci_kernel(const NpciParams p) {
  const int64_t h = blockIdx.y, b = blockIdx.z;
  const int g = threadIdx.x & 15;
  for (int grp = 0; grp < kRowGroups; ++grp) {
    const int64_t row = ((int64_t)blockIdx.x * kRowGroups + grp) * 16 + threadIdx.x / 16;
    npci_row<T>(p, b, h, row < p.N ? row : p.N - 1, row < p.N, g);
  }
}

}  // namespace
}  // namespace dwarf

using namespace dwarf;

extern "C" int dwarf_npci_rotate(const dwarf_npci_rotate_args* a, void* stream) {
  DWARF_CHECK_VERSION(a);
  if (a->dtype != DWARF_BF16 && a->dtype != DWARF_F32) return DWARF_ERR_DTYPE;
  if (a->B < 0 || a->H <= 0 || a->N < 0) return DWARF_ERR_SHAPE;
  if (a->B == 0 || a->N == 0) return DWARF_OK;
  if (!a->x || !a->out || (a->delta && !a->theta)) return DWARF_ERR_NULL;
  if (!(a->tau > 0.0f)) return DWARF_ERR_VALUE;
  NpciParams p{a->B, a->H, a->N, a->x, a->sxb, a->sxh, a->sxn, a->addend, a->sab, a->sah, a->san,
               a->delta, a->sdb, a->sdh, a->sdn, a->theta, a->tau, a->out, a->sob, a->soh, a->son};
  const int64_t per_cta = 16 * kRowGroups;
  if (a->H > 65535 || a->B > 65535 || (a->N + per_cta - 1) / per_cta > 0x7fffffffLL) return DWARF_ERR_SHAPE;
  auto al16 = [](const void* q) { return q == nullptr || (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  const bool vec8 = a->dtype == DWARF_BF16 && al16(a->x) && al16(a->addend) && al16(a->delta) && al16(a->out) &&
                    (a->sxb | a->sxh | a->sxn | a->sob | a->soh | a->son) % 8 == 0 &&
                    (a->addend == nullptr || (a->sab | a->sah | a->san) % 8 == 0) &&
                    (a->delta == nullptr || (a->sdb | a->sdh | a->sdn) % 8 == 0);
  if (vec8) {
    const int64_t rows_per_cta = 32 * kRowGroups;
    const dim3 blocks((unsigned)((a->N + rows_per_cta - 1) / rows_per_cta), (unsigned)a->H, (unsigned)a->B);
    npci_vec8_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(p);
    return launch_status();
  }
  const dim3 blocks((unsigned)((a->N + per_cta - 1) / per_cta), (unsigned)a->H, (unsigned)a->B);
  if (a->dtype == DWARF_BF16)
    npci_kernel<__nv_bfloat16><<<blocks, 256, 0, (cudaStream_t)stream>>>(p);
  else
    npci_kernel<float><<<blocks, 256, 0, (cudaStream_t)stream>>>(p);
  return launch_status();
}
