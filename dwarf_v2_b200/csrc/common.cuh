// Shared device/host helpers for the DWARF-v2 B200 engine (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include "../../include/dwarf_b200.h"

#define DWARF_CHECK_VERSION(a)                                   \
  do {                                                           \
    if ((a) == nullptr) return DWARF_ERR_NULL;                   \
    if ((a)->version != DWARF_ABI_VERSION) return DWARF_ERR_VERSION; \
  } while (0)

namespace dwarf {

constexpr int kNumSMs = 148;

// Bounded spin: about 2^22 polls with a 64 ns back-off (~0.3-1 s) before a
// waiting CTA gives up and records DWARF_DEVICE_TIMEOUT.
constexpr uint32_t kSpinLimit = 1u << 22;

// Status of the last launch; with DWARF_DEBUG set, the CUDA error text goes to stderr.
inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess && getenv("DWARF_DEBUG") != nullptr)
    fprintf(stderr, "dwarf_b200: launch failed: %s\n", cudaGetErrorString(e));
  return e == cudaSuccess ? DWARF_OK : DWARF_ERR_LAUNCH;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ float bf16_to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

// Round-to-nearest-even fp32 -> bf16 (matches torch's .to(torch.bfloat16)).
__device__ __forceinline__ __nv_bfloat16 f32_to_bf16(float v) { return __float2bfloat16_rn(v); }

__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// 2^x on the SFU (ex2.approx; results below 2^-126 flush to zero, 2^-inf = 0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Vector load/store of VEC consecutive elements as fp32.
template <typename T, int VEC>
struct VecIO;

template <>
struct VecIO<float, 1> {
  __device__ __forceinline__ static void load(const float* p, float* o) { o[0] = *p; }
  __device__ __forceinline__ static void store(float* p, const float* v) { *p = v[0]; }
};
template <>
struct VecIO<float, 4> {
  __device__ __forceinline__ static void load(const float* p, float* o) {
    float4 t = *reinterpret_cast<const float4*>(p);
    o[0] = t.x; o[1] = t.y; o[2] = t.z; o[3] = t.w;
  }
  __device__ __forceinline__ static void store(float* p, const float* v) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
};
template <>
struct VecIO<__nv_bfloat16, 1> {
  __device__ __forceinline__ static void load(const __nv_bfloat16* p, float* o) { o[0] = __bfloat162float(*p); }
  __device__ __forceinline__ static void store(__nv_bfloat16* p, const float* v) { *p = __float2bfloat16_rn(v[0]); }
};
template <>
struct VecIO<__nv_bfloat16, 8> {
  __device__ __forceinline__ static void load(const __nv_bfloat16* p, float* o) {
    uint4 t = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&t);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(h[i]);
      o[2 * i] = f.x; o[2 * i + 1] = f.y;
    }
  }
  __device__ __forceinline__ static void store(__nv_bfloat16* p, const float* v) {
    uint4 t;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&t);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = t;
  }
};

}  // namespace dwarf
