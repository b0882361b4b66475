// q6 KV codec: 64-value rows -> 48 bytes of 6-bit codes + one fp16 scale.
//
// The format is defined by this engine (the reference has no packed KV path;
// kernels/dsqg_attention_v22.py:467,473-476 declares it unimplemented):
//   amax = max_d |x_d| (fp32); s = fp16(min(amax, 65504)) (RNE);
//   c_d  = clamp(rint(x_d * (31 / float(s))), -31, 31) (RNE, IEEE div once per row; s == 0 -> 0);
//   group g of 4 codes -> 3 bytes little-endian of w = u0 | u1<<6 | u2<<12 | u3<<18,
//   u = c & 63; dequant x^ = float(c) * (float(s) / 31).
// 16 threads own one row, 4 values (one 3-byte group) each; the row maximum
// is a 16-lane shuffle reduction.
#include "common.cuh"

#include "q6_format.cuh"

namespace dwarf {
namespace {

template <typename T>
__global__ void q6_pack_kernel(const T* __restrict__ x, int64_t B, int64_t H, int64_t T_, int64_t sxb,
                               int64_t sxh, int64_t sxt, uint8_t* __restrict__ codes, int64_t scb,
                               int64_t sch, int64_t sct, uint16_t* __restrict__ scales, int64_t ssb,
                               int64_t ssh, int64_t sst) {
  const int64_t rows = B * H * T_;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 16) + threadIdx.x / 16;
  const int g = threadIdx.x & 15;
  const bool active = row < rows;
  const int64_t r = active ? row : 0;
  const int64_t t = r % T_;
  const int64_t h = (r / T_) % H;
  const int64_t b = r / (T_ * H);
  float v[4] = {0.f, 0.f, 0.f, 0.f};
  if (active) {
    const T* src = x + b * sxb + h * sxh + t * sxt + g * 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = static_cast<float>(src[i]);
  }
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o, 16));
  const __half s = q6_scale_from_amax(amax);
  const float inv = q6_inv_step(__half2float(s));
  uint32_t w = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) w |= (uint32_t)(q6_quantize(v[i], inv) & 63) << (6 * i);
  if (active) {
    uint8_t* dst = codes + b * scb + h * sch + t * sct + g * 3;
    dst[0] = (uint8_t)(w & 255u);
    dst[1] = (uint8_t)((w >> 8) & 255u);
    dst[2] = (uint8_t)((w >> 16) & 255u);
    if (g == 0) scales[b * ssb + h * ssh + t * sst] = __half_as_ushort(s);
  }
}

template <typename T>
__global__ void q6_unpack_kernel(const uint8_t* __restrict__ codes, int64_t B, int64_t H, int64_t T_,
                                 int64_t scb, int64_t sch, int64_t sct, const uint16_t* __restrict__ scales,
                                 int64_t ssb, int64_t ssh, int64_t sst, T* __restrict__ x, int64_t sxb,
                                 int64_t sxh, int64_t sxt) {
  const int64_t rows = B * H * T_;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 16) + threadIdx.x / 16;
  const int g = threadIdx.x & 15;
  if (row >= rows) return;
  const int64_t t = row % T_;
  const int64_t h = (row / T_) % H;
  const int64_t b = row / (T_ * H);
  const uint8_t* src = codes + b * scb + h * sch + t * sct + g * 3;
  const uint32_t w = (uint32_t)src[0] | ((uint32_t)src[1] << 8) | ((uint32_t)src[2] << 16);
  const float step = q6_step(__ushort_as_half(scales[b * ssb + h * ssh + t * sst]));
  T* dst = x + b * sxb + h * sxh + t * sxt + g * 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[i] = static_cast<T>((float)q6_code(w, 6 * i) * step);
}

// ---- vectorised fast path: 4 threads per row, 16 values (12 code bytes) each.
// Rows are (t, bh) with bh = b * H + h from a grid-stride loop on blockIdx.y, so
// no 64-bit division; loads and stores are 16-byte (values) and 4-byte (codes)
// vectors, and the 48-byte code rows of a warp's 8 rows are contiguous when the
// codes tensor is. Requires 16-byte aligned value rows and 4-byte aligned code rows.
constexpr int kVecRows = 64;  // rows per 256-thread CTA

template <typename T>
__device__ __forceinline__ void load16(const T* src, float (&v)[16]);
template <>
__device__ __forceinline__ void load16<__nv_bfloat16>(const __nv_bfloat16* src, float (&v)[16]) {
  const uint4 a = *reinterpret_cast<const uint4*>(src), b = *reinterpret_cast<const uint4*>(src + 8);
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
template <>
__device__ __forceinline__ void load16<float>(const float* src, float (&v)[16]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 f = reinterpret_cast<const float4*>(src)[i];
    v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
  }
}

template <typename T>
__device__ __forceinline__ void store16(T* dst, const float (&v)[16]);
template <>
__device__ __forceinline__ void store16<__nv_bfloat16>(__nv_bfloat16* dst, const float (&v)[16]) {
  uint32_t w[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&p);
  }
  reinterpret_cast<uint4*>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
  reinterpret_cast<uint4*>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
}
template <>
__device__ __forceinline__ void store16<float>(float* dst, const float (&v)[16]) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
    reinterpret_cast<float4*>(dst)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

template <typename T>
__global__ void __launch_bounds__(256) q6_pack_vec_kernel(const T* __restrict__ x, int64_t BH, int64_t H, int64_t T_,
                                                          int64_t sxb, int64_t sxh, int64_t sxt,
                                                          uint8_t* __restrict__ codes, int64_t scb, int64_t sch,
                                                          int64_t sct, uint16_t* __restrict__ scales, int64_t ssb,
                                                          int64_t ssh, int64_t sst) {
  const int q = threadIdx.x & 3;
  const int64_t t = (int64_t)blockIdx.x * kVecRows + (threadIdx.x >> 2);
  for (int64_t bh = blockIdx.y; bh < BH; bh += gridDim.y) {
    const int64_t b = bh / H, h = bh - b * H;  // once per CTA row pass, not per element
    float v[16];
    if (t < T_) load16<T>(x + b * sxb + h * sxh + t * sxt + q * 16, v);
    else
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = 0.f;
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const __half s = q6_scale_from_amax(amax);
    const float inv = q6_inv_step(__half2float(s));
    const bool clamp = q6_needs_clamp(amax, inv);
    uint32_t g[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      g[j] = 0;
      if (!clamp) {
#pragma unroll
        for (int i = 0; i < 4; ++i) g[j] |= q6_bits(v[4 * j + i], inv, false) << (6 * i);
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) g[j] |= q6_bits(v[4 * j + i], inv, true) << (6 * i);
      }
    }
    if (t < T_) {
      // four 24-bit groups -> three little-endian 32-bit words
      uint32_t* dst = reinterpret_cast<uint32_t*>(codes + b * scb + h * sch + t * sct + q * 12);
      dst[0] = g[0] | (g[1] << 24);
      dst[1] = (g[1] >> 8) | (g[2] << 16);
      dst[2] = (g[2] >> 16) | (g[3] << 8);
      if (q == 0) scales[b * ssb + h * ssh + t * sst] = __half_as_ushort(s);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) q6_unpack_vec_kernel(const uint8_t* __restrict__ codes, int64_t BH, int64_t H,
                                                            int64_t T_, int64_t scb, int64_t sch, int64_t sct,
                                                            const uint16_t* __restrict__ scales, int64_t ssb,
                                                            int64_t ssh, int64_t sst, T* __restrict__ x, int64_t sxb,
                                                            int64_t sxh, int64_t sxt) {
  const int q = threadIdx.x & 3;
  const int64_t t = (int64_t)blockIdx.x * kVecRows + (threadIdx.x >> 2);
  if (t >= T_) return;
  for (int64_t bh = blockIdx.y; bh < BH; bh += gridDim.y) {
    const int64_t b = bh / H, h = bh - b * H;
    const uint32_t* src = reinterpret_cast<const uint32_t*>(codes + b * scb + h * sch + t * sct + q * 12);
    const uint32_t w0 = src[0], w1 = src[1], w2 = src[2];
    const uint32_t g[4] = {w0 & 0xffffffu, (w0 >> 24) | ((w1 & 0xffffu) << 8), (w1 >> 16) | ((w2 & 0xffu) << 16),
                           w2 >> 8};
    const float step = q6_step(__ushort_as_half(scales[b * ssb + h * ssh + t * sst]));
    float v[16];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int i = 0; i < 4; ++i) v[4 * j + i] = (float)q6_code(g[j], 6 * i) * step;
    store16<T>(x + b * sxb + h * sxh + t * sxt + q * 16, v);
  }
}

inline bool vec_ok(const void* values, int64_t elem, int64_t sb, int64_t sh, int64_t st, const void* codes,
                   int64_t cb, int64_t ch, int64_t ct) {
  return aligned16(values) && ((sb * elem) & 15) == 0 && ((sh * elem) & 15) == 0 && ((st * elem) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(codes) & 3u) == 0 && (cb & 3) == 0 && (ch & 3) == 0 && (ct & 3) == 0;
}

inline dim3 vec_grid(int64_t BH, int64_t T_) {
  const int64_t y = BH < 65535 ? BH : 65535;
  return dim3((unsigned)((T_ + kVecRows - 1) / kVecRows), (unsigned)y);
}

}  // namespace
}  // namespace dwarf

using namespace dwarf;

extern "C" int dwarf_q6_pack(const dwarf_q6_pack_args* a, void* stream) {
  DWARF_CHECK_VERSION(a);
  if (a->dtype != DWARF_BF16 && a->dtype != DWARF_F32) return DWARF_ERR_DTYPE;
  if (a->B < 0 || a->H < 0 || a->T < 0) return DWARF_ERR_SHAPE;
  const int64_t rows = a->B * a->H * a->T;
  if (rows == 0) return DWARF_OK;
  if (!a->x || !a->codes || !a->scales) return DWARF_ERR_NULL;
  const int64_t elem = a->dtype == DWARF_BF16 ? 2 : 4;
  if (vec_ok(a->x, elem, a->sxb, a->sxh, a->sxt, a->codes, a->scb, a->sch, a->sct) &&
      (a->T + kVecRows - 1) / kVecRows <= 2147483647LL) {
    const dim3 grid = vec_grid(a->B * a->H, a->T);
    if (a->dtype == DWARF_BF16)
      q6_pack_vec_kernel<__nv_bfloat16><<<grid, 256, 0, (cudaStream_t)stream>>>(
          (const __nv_bfloat16*)a->x, a->B * a->H, a->H, a->T, a->sxb, a->sxh, a->sxt, a->codes, a->scb, a->sch,
          a->sct, a->scales, a->ssb, a->ssh, a->sst);
    else
      q6_pack_vec_kernel<float><<<grid, 256, 0, (cudaStream_t)stream>>>(
          (const float*)a->x, a->B * a->H, a->H, a->T, a->sxb, a->sxh, a->sxt, a->codes, a->scb, a->sch, a->sct,
          a->scales, a->ssb, a->ssh, a->sst);
    return launch_status();
  }
  const unsigned blocks = (unsigned)((rows + 15) / 16);
  if (a->dtype == DWARF_BF16) {
    q6_pack_kernel<__nv_bfloat16><<<blocks, 256, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16*)a->x, a->B, a->H, a->T, a->sxb, a->sxh, a->sxt, a->codes, a->scb, a->sch,
        a->sct, a->scales, a->ssb, a->ssh, a->sst);
  } else {
    q6_pack_kernel<float><<<blocks, 256, 0, (cudaStream_t)stream>>>(
        (const float*)a->x, a->B, a->H, a->T, a->sxb, a->sxh, a->sxt, a->codes, a->scb, a->sch, a->sct,
        a->scales, a->ssb, a->ssh, a->sst);
  }
  return launch_status();
}

extern "C" int dwarf_q6_unpack(const dwarf_q6_unpack_args* a, void* stream) {
  DWARF_CHECK_VERSION(a);
  if (a->out_dtype != DWARF_BF16 && a->out_dtype != DWARF_F32) return DWARF_ERR_DTYPE;
  if (a->B < 0 || a->H < 0 || a->T < 0) return DWARF_ERR_SHAPE;
  const int64_t rows = a->B * a->H * a->T;
  if (rows == 0) return DWARF_OK;
  if (!a->x || !a->codes || !a->scales) return DWARF_ERR_NULL;
  const int64_t elem = a->out_dtype == DWARF_BF16 ? 2 : 4;
  if (vec_ok(a->x, elem, a->sxb, a->sxh, a->sxt, a->codes, a->scb, a->sch, a->sct) &&
      (a->T + kVecRows - 1) / kVecRows <= 2147483647LL) {
    const dim3 grid = vec_grid(a->B * a->H, a->T);
    if (a->out_dtype == DWARF_BF16)
      q6_unpack_vec_kernel<__nv_bfloat16><<<grid, 256, 0, (cudaStream_t)stream>>>(
          a->codes, a->B * a->H, a->H, a->T, a->scb, a->sch, a->sct, a->scales, a->ssb, a->ssh, a->sst,
          (__nv_bfloat16*)a->x, a->sxb, a->sxh, a->sxt);
    else
      q6_unpack_vec_kernel<float><<<grid, 256, 0, (cudaStream_t)stream>>>(
          a->codes, a->B * a->H, a->H, a->T, a->scb, a->sch, a->sct, a->scales, a->ssb, a->ssh, a->sst,
          (float*)a->x, a->sxb, a->sxh, a->sxt);
    return launch_status();
  }
  const unsigned blocks = (unsigned)((rows + 15) / 16);
  if (a->out_dtype == DWARF_BF16) {
    q6_unpack_kernel<__nv_bfloat16><<<blocks, 256, 0, (cudaStream_t)stream>>>(
        a->codes, a->B, a->H, a->T, a->scb, a->sch, a->sct, a->scales, a->ssb, a->ssh, a->sst,
        (__nv_bfloat16*)a->x, a->sxb, a->sxh, a->sxt);
  } else {
    q6_unpack_kernel<float><<<blocks, 256, 0, (cudaStream_t)stream>>>(
        a->codes, a->B, a->H, a->T, a->scb, a->sch, a->sct, a->scales, a->ssb, a->ssh, a->sst, (float*)a->x,
        a->sxb, a->sxh, a->sxt);
  }
  return launch_status();
}
