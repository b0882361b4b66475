// Row-wise block glue of the DWARF-v2 blocks, each a single pass over HBM.
//
// The reference runs these as separate ATen/Inductor passes
// (train/train_dwarf.py:218-240 RMSNorm/SwiGLU, 260-284 InterferencePacket,
// 320-322 / 356-364 residual adds, 439-447 embedding). Here:
//   dwarf_add_rmsnorm   residual add (+ optional sigmoid-gated addend) fused
//                       with the following RMSNorm
//   dwarf_embed_rmsnorm embedding gather fused with the first RMSNorm
//   dwarf_swiglu        silu(gate) * up
//   dwarf_gate_mul      a * sigmoid(g)
//   dwarf_packet        the EMA-packet epilogue (mixture, RMS direction,
//                       confidence, gate)
// Each op keeps the reference's bf16 rounding points so results track the
// bf16 reference step for step.
#include "common.cuh"

#include <algorithm>

namespace dwarf {
namespace {

constexpr int kMaxWidth = 1024;
constexpr int kSeg = 256;  // values per warp-wide 16-byte access

__device__ __forceinline__ void ld8(const __nv_bfloat16* p, float (&v)[8]) { VecIO<__nv_bfloat16, 8>::load(p, v); }
__device__ __forceinline__ void unpack8(const uint4& w, float (&v)[8]) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(u[i] << 16);
    v[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
  }
}
__device__ __forceinline__ void st8(__nv_bfloat16* p, const float (&v)[8]) { VecIO<__nv_bfloat16, 8>::store(p, v); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }

template <int NSEG>
__device__ __forceinline__ void load_weight(const void* w, int w_bf16, int lane, float (&out)[NSEG][8]) {
#pragma unroll
  for (int s = 0; s < NSEG; ++s) {
    const int c = s * kSeg + lane * 8;
    if (w_bf16) {
      ld8(static_cast<const __nv_bfloat16*>(w) + c, out[s]);
    } else {
      const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(w) + c);
      const float4 a = p[0], b = p[1];
      out[s][0] = a.x; out[s][1] = a.y; out[s][2] = a.z; out[s][3] = a.w;
      out[s][4] = b.x; out[s][5] = b.y; out[s][6] = b.z; out[s][7] = b.w;
    }
  }
}

// RMSNorm of the row held in v, written to n as the reference computes it:
// (x * rsqrt(mean(x^2) + eps)) * w in fp32, one rounding to bf16.
template <int NSEG>
__device__ __forceinline__ void rmsnorm_store(const float (&v)[NSEG][8], const float (&w)[NSEG][8], float eps,
                                              int width, __nv_bfloat16* n, int lane) {
  float ss = 0.0f;
#pragma unroll
  for (int s = 0; s < NSEG; ++s)
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += v[s][i] * v[s][i];
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)width + eps);
#pragma unroll
  for (int s = 0; s < NSEG; ++s) {
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = (v[s][i] * r) * w[s][i];
    st8(n + s * kSeg + lane * 8, o);
  }
}

template <int NSEG>
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(dwarf_add_rmsnorm_args a) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= a.rows) return;
  float v[NSEG][8];
  const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(a.x) + row * a.sx;
#pragma unroll
  for (int s = 0; s < NSEG; ++s) ld8(x + s * kSeg + lane * 8, v[s]);
  if (a.a != nullptr) {
    const __nv_bfloat16* ad = static_cast<const __nv_bfloat16*>(a.a) + row * a.sa;
    const __nv_bfloat16* gt = a.g ? static_cast<const __nv_bfloat16*>(a.g) + row * a.sg : nullptr;
#pragma unroll
    for (int s = 0; s < NSEG; ++s) {
      float t[8];
      ld8(ad + s * kSeg + lane * 8, t);
      if (gt != nullptr) {
        float gv[8];
        ld8(gt + s * kSeg + lane * 8, gv);
#pragma unroll
        for (int i = 0; i < 8; ++i) t[i] = round_bf16(t[i] * round_bf16(sigmoid_f(gv[i])));
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) v[s][i] = round_bf16(v[s][i] + t[i]);
    }
  }
  if (a.x_out != nullptr) {
    __nv_bfloat16* xo = static_cast<__nv_bfloat16*>(a.x_out) + row * a.sxo;
#pragma unroll
    for (int s = 0; s < NSEG; ++s) st8(xo + s * kSeg + lane * 8, v[s]);
  }
  float w[NSEG][8];
  load_weight<NSEG>(a.w, a.w_dtype == DWARF_BF16, lane, w);
  rmsnorm_store<NSEG>(v, w, a.eps, (int)a.width, static_cast<__nv_bfloat16*>(a.n_out) + row * a.sno, lane);
}

template <int NSEG>
__global__ void __launch_bounds__(256) embed_rmsnorm_kernel(dwarf_embed_rmsnorm_args a) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= a.rows) return;
  int64_t id = a.ids[row];
  id = id < 0 ? 0 : (id >= a.vocab ? a.vocab - 1 : id);  // callers validate ids
  const __nv_bfloat16* e = static_cast<const __nv_bfloat16*>(a.embedding) + id * a.width;
  float v[NSEG][8];
#pragma unroll
  for (int s = 0; s < NSEG; ++s) ld8(e + s * kSeg + lane * 8, v[s]);
  __nv_bfloat16* xo = static_cast<__nv_bfloat16*>(a.x_out) + row * a.width;
#pragma unroll
  for (int s = 0; s < NSEG; ++s) st8(xo + s * kSeg + lane * 8, v[s]);
  float w[NSEG][8];
  load_weight<NSEG>(a.w, a.w_dtype == DWARF_BF16, lane, w);
  rmsnorm_store<NSEG>(v, w, a.eps, (int)a.width, static_cast<__nv_bfloat16*>(a.n_out) + row * a.width, lane);
}

// 8 outputs per thread, grid-stride over rows * hidden/8.
__global__ void __launch_bounds__(256) swiglu_kernel(dwarf_swiglu_args a) {
  const int64_t per_row = a.hidden / 8;
  const int64_t total = a.rows * per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / per_row, c = (i % per_row) * 8;
    const __nv_bfloat16* in = static_cast<const __nv_bfloat16*>(a.in) + r * a.sin;
    float up[8], gate[8], o[8];
    ld8(in + c, up);
    ld8(in + a.hidden + c, gate);
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = round_bf16(gate[k] / (1.0f + expf(-gate[k]))) * up[k];
    st8(static_cast<__nv_bfloat16*>(a.out) + r * a.sout + c, o);
  }
}

__global__ void __launch_bounds__(256) gate_mul_kernel(dwarf_gate_mul_args a) {
  const int64_t per_row = a.width / 8;
  const int64_t total = a.rows * per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / per_row, c = (i % per_row) * 8;
    float x[8], g[8], o[8];
    ld8(static_cast<const __nv_bfloat16*>(a.a) + r * a.sa + c, x);
    ld8(static_cast<const __nv_bfloat16*>(a.g) + r * a.sg + c, g);
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = x[k] * round_bf16(sigmoid_f(g[k]));
    st8(static_cast<__nv_bfloat16*>(a.out) + r * a.so + c, o);
  }
}

template <int NSEG>
__global__ void __launch_bounds__(256) packet_kernel(dwarf_packet_args a) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= a.rows) return;
  // Every load of the row (all scans, then the gate) is issued before any
  // arithmetic, as raw 16-byte words.
  uint4 raw[3][NSEG], graw[NSEG];
  const __nv_bfloat16* gp = static_cast<const __nv_bfloat16*>(a.gate_pre) + row * a.sgp;
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    if (k < a.n_scans) {
      const __nv_bfloat16* sc = static_cast<const __nv_bfloat16*>(a.scans[k]) + row * a.sscan;
#pragma unroll
      for (int s = 0; s < NSEG; ++s) raw[k][s] = *reinterpret_cast<const uint4*>(sc + s * kSeg + lane * 8);
    }
  }
#pragma unroll
  for (int s = 0; s < NSEG; ++s) graw[s] = *reinterpret_cast<const uint4*>(gp + s * kSeg + lane * 8);
  float pooled[NSEG][8];
#pragma unroll
  for (int s = 0; s < NSEG; ++s)
#pragma unroll
    for (int i = 0; i < 8; ++i) pooled[s][i] = 0.0f;
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    if (k < a.n_scans) {
      const float wk = a.mix[k];
#pragma unroll
      for (int s = 0; s < NSEG; ++s) {
        float t[8];
        unpack8(raw[k][s], t);
#pragma unroll
        for (int i = 0; i < 8; ++i) pooled[s][i] = round_bf16(pooled[s][i] + round_bf16(wk * t[i]));
      }
    }
  }
  float ss = 0.0f;
#pragma unroll
  for (int s = 0; s < NSEG; ++s)
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += pooled[s][i] * pooled[s][i];
  const float ms = warp_sum(ss) / (float)a.width;
  const float conf = tanhf(sqrtf(ms) / 0.25f);
  const float rs = rsqrtf(ms + 1e-6f);
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out) + row * a.so;
#pragma unroll
  for (int s = 0; s < NSEG; ++s) {
    float g[8], o[8];
    unpack8(graw[s], g);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = ((pooled[s][i] * rs) * conf) * sigmoid_f(g[i]);
    st8(out + s * kSeg + lane * 8, o);
  }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool width_ok(int64_t w) { return w > 0 && w % kSeg == 0 && w <= kMaxWidth; }

}  // namespace
}  // namespace dwarf

using namespace dwarf;

#define DWARF_ROWS_DISPATCH(KERNEL, ARGS, ROWS, WIDTH, STREAM)      \
  do {                                                              \
    const unsigned blocks_ = (unsigned)(((ROWS) + 7) / 8);          \
    switch ((WIDTH) / kSeg) {                                       \
      case 1: KERNEL<1><<<blocks_, 256, 0, STREAM>>>(ARGS); break; \
      case 2: KERNEL<2><<<blocks_, 256, 0, STREAM>>>(ARGS); break; \
      case 3: KERNEL<3><<<blocks_, 256, 0, STREAM>>>(ARGS); break; \
      case 4: KERNEL<4><<<blocks_, 256, 0, STREAM>>>(ARGS); break; \
      default: return DWARF_ERR_SHAPE;                              \
    }                                                               \
  } while (0)

extern "C" int dwarf_add_rmsnorm(const dwarf_add_rmsnorm_args* a, void* stream) {
  DWARF_CHECK_VERSION(a);
  if (!width_ok(a->width) || a->rows < 0) return DWARF_ERR_SHAPE;
  if (a->rows == 0) return DWARF_OK;
  if (!a->x || !a->w || !a->n_out || (a->g && !a->a)) return DWARF_ERR_NULL;
  if (a->w_dtype != DWARF_F32 && a->w_dtype != DWARF_BF16) return DWARF_ERR_DTYPE;
  if (!al16(a->x) || !al16(a->n_out) || !al16(a->w) || (a->a && !al16(a->a)) || (a->g && !al16(a->g)) ||
      (a->x_out && !al16(a->x_out)) || (a->sx | a->sno | a->sa | a->sg | a->sxo) % 8 != 0)
    return DWARF_ERR_ALIGN;
  if (a->rows / 8 + 1 > 0x7fffffffLL) return DWARF_ERR_SHAPE;
  DWARF_ROWS_DISPATCH(add_rmsnorm_kernel, *a, a->rows, a->width, (cudaStream_t)stream);
  return launch_status();
}

extern "C" int dwarf_embed_rmsnorm(const dwarf_embed_rmsnorm_args* a, void* stream) {
  DWARF_CHECK_VERSION(a);
  if (!width_ok(a->width) || a->rows < 0 || a->vocab <= 0) return DWARF_ERR_SHAPE;
  if (a->rows == 0) return DWARF_OK;
  if (!a->ids || !a->embedding || !a->w || !a->x_out || !a->n_out) return DWARF_ERR_NULL;
  if (a->w_dtype != DWARF_F32 && a->w_dtype != DWARF_BF16) return DWARF_ERR_DTYPE;
  if (!al16(a->embedding) || !al16(a->w) || !al16(a->x_out) || !al16(a->n_out)) return DWARF_ERR_ALIGN;
  DWARF_ROWS_DISPATCH(embed_rmsnorm_kernel, *a, a->rows, a->width, (cudaStream_t)stream);
  return launch_status();
}

extern "C" int dwarf_swiglu(const dwarf_swiglu_args* a, void* stream) {
  DWARF_CHECK_VERSION(a);
  if (a->rows < 0 || a->hidden <= 0 || a->hidden % 8 != 0) return DWARF_ERR_SHAPE;
  if (a->rows == 0) return DWARF_OK;
  if (!a->in || !a->out) return DWARF_ERR_NULL;
  if (!al16(a->in) || !al16(a->out) || (a->sin | a->sout) % 8 != 0) return DWARF_ERR_ALIGN;
  const int64_t total = a->rows * (a->hidden / 8);
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, (int64_t)kNumSMs * 16);
  swiglu_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(*a);
  return launch_status();
}

extern "C" int dwarf_gate_mul(const dwarf_gate_mul_args* a, void* stream) {
  DWARF_CHECK_VERSION(a);
  if (a->rows < 0 || a->width <= 0 || a->width % 8 != 0) return DWARF_ERR_SHAPE;
  if (a->rows == 0) return DWARF_OK;
  if (!a->a || !a->g || !a->out) return DWARF_ERR_NULL;
  if (!al16(a->a) || !al16(a->g) || !al16(a->out) || (a->sa | a->sg | a->so) % 8 != 0) return DWARF_ERR_ALIGN;
  const int64_t total = a->rows * (a->width / 8);
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, (int64_t)kNumSMs * 16);
  gate_mul_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(*a);
  return launch_status();
}

extern "C" int dwarf_packet(const dwarf_packet_args* a, void* stream) {
  DWARF_CHECK_VERSION(a);
  if (!width_ok(a->width) || a->rows < 0 || a->n_scans < 1 || a->n_scans > 3) return DWARF_ERR_SHAPE;
  if (a->rows == 0) return DWARF_OK;
  for (int k = 0; k < a->n_scans; ++k)
    if (!a->scans[k] || !al16(a->scans[k])) return a->scans[k] ? DWARF_ERR_ALIGN : DWARF_ERR_NULL;
  if (!a->gate_pre || !a->out) return DWARF_ERR_NULL;
  if (!al16(a->gate_pre) || !al16(a->out) || (a->sscan | a->sgp | a->so) % 8 != 0) return DWARF_ERR_ALIGN;
  DWARF_ROWS_DISPATCH(packet_kernel, *a, a->rows, a->width, (cudaStream_t)stream);
  return launch_status();
}
