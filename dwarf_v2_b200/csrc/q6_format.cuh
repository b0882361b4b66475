// q6 format primitives shared by the codec, the QKV prep kernel and the
// DSQG kernel (the format is specified in include/dwarf_b200.h).
#pragma once

#include "common.cuh"

namespace dwarf {

// fp16 scale of a row from its absolute maximum.
__device__ __forceinline__ __half q6_scale_from_amax(float amax) {
  return __float2half_rn(fminf(amax, 65504.0f));
}

// Per-row quantisation factor 31 / float(s) (IEEE division); 0 when s == 0.
__device__ __forceinline__ float q6_inv_step(float s) { return s > 0.0f ? __fdiv_rn(31.0f, s) : 0.0f; }

// Code of one value: clamp(rint(x * inv), -31, 31), inv = q6_inv_step(s).
__device__ __forceinline__ int q6_quantize(float x, float inv) {
  float q = rintf(__fmul_rn(x, inv));
  q = fminf(fmaxf(q, -31.0f), 31.0f);
  return (int)q;
}

// The low six bits of the code of x (two's complement), as q6_quantize: adding
// 1.5 * 2^23 to the (clamped) product rounds it to nearest-even into the low
// mantissa bits. `clamp` may be false only when fmul_rn(amax, inv) < 31.5 for
// the row's amax: rounding is monotonic, so no product then reaches 31.5 and the
// clamp is the identity. Multiply and add stay separate IEEE operations (a fused
// pair rounds once and can resolve a .5 tie differently).
__device__ __forceinline__ uint32_t q6_bits(float x, float inv, bool clamp) {
  float q = __fmul_rn(x, inv);
  if (clamp) q = fminf(fmaxf(q, -31.0f), 31.0f);
  return __float_as_uint(__fadd_rn(q, 12582912.0f)) & 63u;
}
__device__ __forceinline__ bool q6_needs_clamp(float amax, float inv) { return !(__fmul_rn(amax, inv) < 31.5f); }

// Dequantisation step float(s) / 31 (IEEE division).
__device__ __forceinline__ float q6_step(__half s) { return __fdiv_rn(__half2float(s), 31.0f); }

// Signed 6-bit code starting at bit `bit` (< 27) of w.
__device__ __forceinline__ int q6_code(uint32_t w, int bit) {
  return (int)(w << (26 - bit)) >> 26;
}

// Signed 6-bit code i (0..15) of a 96-bit little-endian stream w[0..2].
template <int I>
__device__ __forceinline__ int q6_code96(const uint32_t (&w)[3]) {
  constexpr int bit = 6 * I;
  constexpr int word = bit >> 5;
  constexpr int off = bit & 31;
  if constexpr (off <= 26) {
    return (int)(w[word] << (26 - off)) >> 26;
  } else {
    const uint32_t u = __funnelshift_r(w[word], w[word + 1], off);
    return (int)(u << 26) >> 26;
  }
}

}  // namespace dwarf
