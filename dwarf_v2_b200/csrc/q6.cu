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
