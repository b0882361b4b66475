// Shared pieces of the two DSQG forward kernels (dsqg_fwd.cu: row gathers
// from global memory, any layout; dsqg_resident.cu: the whole q6 K/V of one
// (batch, head) resident in shared memory): launch parameters and the q6
// decode helpers.
#pragma once

#include "common.cuh"
#include "q6_format.cuh"

namespace dwarf {
namespace dsqg {

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
  int32_t* status;  // optional device status word (DWARF_DEVICE_TIMEOUT)
  int64_t row_begin;  // first query row computed (gather kernel)
  const int64_t* pos;  // optional device row_begin (decode kernel)
  int round_split;      // resident kernel with gridDim.z == 2: CTA z = 0 takes the query
                        // rounds [round_split, end), z = 1 the rounds [0, round_split)
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

// q6 row slice of one thread (16 codes = 12 bytes) decoded as offset-binary
// u = c + 32 in [1, 63]. XOR-ing bit 5 of every 6-bit field turns two's
// complement into offset binary. Field i is then read in place, scaled by a
// power of two 2^K_i: masking its 6 bits (at bit K_i <= 17, after at most one
// shift of its word) into the mantissa of 2^23 and subtracting 2^23 gives
// u_i * 2^K_i exactly, with one LOP3 and one FADD and no int->float
// conversion. Callers pre-scale q by 2^-K_i (K path) or post-scale the
// accumulator (V path), and remove the +32 bias with one per-row term.
__device__ __forceinline__ void q6_flip_sign_bits(uint32_t (&w)[3]) {
  w[0] ^= 0x20820820u;  // stream bits 5, 11, 17, 23, 29
  w[1] ^= 0x08208208u;  // stream bits 35, 41, 47, 53, 59
  w[2] ^= 0x82082082u;  // stream bits 65, 71, 77, 83, 89, 95
}
// Power-of-two placement K_i of field i (see q6_scaled16).
__host__ __device__ constexpr int q6_field_shift(int i) {
  constexpr int k[16] = {0, 6, 12, 6, 12, 0, 4, 10, 16, 10, 0, 2, 8, 14, 8, 14};
  return k[i];
}
__device__ __forceinline__ float q6_field(uint32_t src, int k) {
  return __int_as_float(0x4B000000u | (src & (63u << k))) - 8388608.0f;
}
// o[i] = u_i * 2^K_i for the 16 codes of a flipped 96-bit slice.
__device__ __forceinline__ void q6_scaled16(const uint32_t (&w)[3], float (&o)[16]) {
  const uint32_t w0s = w[0] >> 12, w1s = w[1] >> 12, w2s = w[2] >> 12;
  const uint32_t f5 = __funnelshift_r(w[0], w[1], 30);
  const uint32_t f10 = __funnelshift_r(w[1], w[2], 28);
  o[0] = q6_field(w[0], 0);   o[1] = q6_field(w[0], 6);   o[2] = q6_field(w[0], 12);
  o[3] = q6_field(w0s, 6);    o[4] = q6_field(w0s, 12);   o[5] = q6_field(f5, 0);
  o[6] = q6_field(w[1], 4);   o[7] = q6_field(w[1], 10);  o[8] = q6_field(w[1], 16);
  o[9] = q6_field(w1s, 10);   o[10] = q6_field(f10, 0);   o[11] = q6_field(w[2], 2);
  o[12] = q6_field(w[2], 8);  o[13] = q6_field(w[2], 14); o[14] = q6_field(w2s, 8);
  o[15] = q6_field(w2s, 14);
}

}  // namespace dsqg

// Resident-K/V DSQG forward (dsqg_resident.cu). Returns DWARF_OK or an error
// status after launching, or kNotApplicable when the problem does not fit its
// layout and size limits (the caller then uses the gather kernel).
constexpr int kNotApplicable = 1;
int dsqg_resident_launch(const dsqg::DsqgParams& p, int64_t B, cudaStream_t stream);

}  // namespace dwarf
