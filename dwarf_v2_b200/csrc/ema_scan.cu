// Causal EMA scan: one-pass chunked scan chained by decoupled look-back.
//
// Replaces the reference's three-launch blocked scan (_fwd_local -> _fwd_carry
// -> _fwd_apply, kernels/causal_ema_scan.py:73-155, launched from
// _CausalEMAFn.forward :265-313), which writes y twice and serialises the
// carry over time blocks in one program per channel block.
//
// Recurrence: y[t] = a*x[t] + d*y[t-1], d = 1 - a, y[-1] = 0, fp32 state.
//
// Decomposition. A "series" is one (batch row, block of C = 32*VEC channels);
// each lane owns VEC adjacent channels and moves them with one 16-byte access
// per token. A tile is one chunk of CH = WARPS*TS consecutive tokens of one
// series; warp w of the CTA scans tokens [w*TS, (w+1)*TS) of the tile.
// Persistent CTAs (cooperative launch, so all are co-resident) take tiles
// round-robin in chunk-major order, and for each tile:
//   1. stage the tile's x in shared memory (cp.async; the next tile is staged
//      while the current one is finished),
//   2. scan each warp's TS tokens from a zero state -> warp end states,
//   3. warp 0 combines them into the tile aggregate, publishes it, walks back
//      over up to LB predecessor tiles of the same series (LB - 1 aggregates
//      + 1 inclusive prefix) to get the carry-in, and publishes the inclusive
//      prefix (LB = 1 with many series in flight: the window costs registers,
//      hence occupancy, and the series themselves hide the chain's latency;
//      LB = 2 with few series),
//   4. each warp rescans its tokens from its true carry-in and writes y once.
//
// Publication without fences: every published channel value travels in one
// 64-bit scalar {value bits, tag}, written and read as one single-copy-atomic
// b64 access, where tag identifies this launch. A reader spins until the
// tag matches, so no __threadfence/flag pair is needed. The launch tag is kept
// in the workspace header: each launch uses tag = header.epoch + 1 and the last
// CTA to exit advances header.epoch, so consecutive launches never see each
// other's records and the workspace needs zero-filling only once, before its
// first use.
//
// Waits are bounded (kSpinLimit polls, or the caller's wait_limit); a timed-out wait records
// DWARF_DEVICE_TIMEOUT and continues with a zero carry instead of hanging.
// Summation order in the look-back is fixed, so results are bitwise
// reproducible run to run.
#include "common.cuh"

#include <algorithm>

namespace dwarf {
namespace {

constexpr int kLookbackFew = 2;   // look-back window with few series in flight
constexpr int kLookbackMany = 1;  // ... and with many (>= kManySeries)
constexpr int64_t kManySeries = 256;

struct EmaWorkspace {
  uint32_t* header;  // [0] epoch, [32] exit counter (separate 128-B lines)
  uint2* agg;        // [ntiles][C] {value bits, tag}
  uint2* incl;       // [ntiles][C]
};

inline int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }
constexpr int64_t kHeaderBytes = 256;

// A record is ONE 64-bit scalar (value bits in the low word, tag in the high
// word), stored and loaded with a single b64 access: the PTX memory model
// makes a scalar access single-copy atomic, whereas the two halves of a
// .v2.u32 access may be observed separately (a new tag with a stale value).
__device__ __forceinline__ void st_rec(uint2* p, float v, uint32_t tag) {
  const unsigned long long w = (unsigned long long)__float_as_uint(v) | ((unsigned long long)tag << 32);
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint2 ld_rec(const uint2* p) {
  unsigned long long w;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return make_uint2((uint32_t)w, (uint32_t)(w >> 32));
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

template <typename T, int VEC>
__device__ __forceinline__ void stage_row(T* smem, const T* gmem, bool valid) {
  if constexpr (VEC * sizeof(T) == 16) {
    const uint32_t saddr = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    const int src_bytes = valid ? 16 : 0;  // 0 => zero-fill
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(saddr), "l"(gmem), "r"(src_bytes)
                 : "memory");
  } else {
#pragma unroll
    for (int v = 0; v < VEC; ++v) smem[v] = valid ? gmem[v] : T(0.0f);
  }
}

template <typename T, int VEC, int TS, int WARPS, int kLookback>
__global__ void __launch_bounds__(WARPS * 32, 1)
ema_scan_lookback_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t seq_len, int64_t width,
                         int64_t sxb, int64_t sxn, int64_t sxd, int64_t syb, int64_t syn, int64_t syd,
                         const float* __restrict__ alpha, int alpha_per_channel, int clamp, float lo,
                         float hi, EmaWorkspace ws, int64_t nseries, int64_t ncb, int64_t ntiles,
                         int32_t* device_status, const float* __restrict__ init_state,
                         float* __restrict__ final_state, uint32_t spin_limit, uint32_t tag_skew) {
  constexpr int C = 32 * VEC;  // channels per series
  constexpr int CH = WARPS * TS;
  constexpr bool kAsync = VEC * sizeof(T) == 16;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* bufs = reinterpret_cast<T*>(smem_raw);  // [2][WARPS][TS][C]
  __shared__ float s_end[WARPS][C];
  __shared__ float s_carry[C];

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(ws.header);
  const uint32_t tag = epoch + 1u;  // never 0 (0 = never written)
  bool timed_out = false;

  auto stage = [&](int64_t tile, int slot) {
    const int64_t chunk = tile / nseries;
    const int64_t series = tile % nseries;
    const int64_t b = series / ncb;
    const int64_t c0 = (series % ncb) * C + (int64_t)lane * VEC;
    const int64_t t0 = chunk * CH + (int64_t)warp * TS;
    const bool active = c0 < width;
    T* my_x = bufs + ((size_t)slot * WARPS * TS + (size_t)warp * TS) * C + lane * VEC;
    const T* xrow = x + b * sxb + t0 * sxn + c0 * sxd;
#pragma unroll
    for (int i = 0; i < TS; ++i) stage_row<T, VEC>(my_x + i * C, xrow + i * sxn, active && t0 + i < seq_len);
  };

  int64_t cur = blockIdx.x;
  if (cur < ntiles) stage(cur, 0);
  if constexpr (kAsync) cp_async_commit();
  int64_t nxt = cur + gridDim.x;
  if (nxt < ntiles) stage(nxt, 1);
  if constexpr (kAsync) cp_async_commit();

  for (int it = 0; cur < ntiles; ++it) {
    const int slot = it & 1;
    const int64_t tile = cur;
    const int64_t chunk = tile / nseries;
    const int64_t series = tile % nseries;
    const int64_t b = series / ncb;
    const int64_t c0 = (series % ncb) * C + (int64_t)lane * VEC;
    const bool lane_active = c0 < width;  // width % VEC == 0 for VEC > 1
    const int64_t t0 = chunk * CH + (int64_t)warp * TS;
    const int64_t rem = seq_len - t0;
    const int nvalid = rem <= 0 ? 0 : (rem >= TS ? TS : (int)rem);
    const T* my_x = bufs + ((size_t)slot * WARPS * TS + (size_t)warp * TS) * C + lane * VEC;

    float a[VEC], d[VEC], dts[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      float av = alpha[alpha_per_channel ? (lane_active ? c0 + v : 0) : 0];
      if (clamp) av = fminf(fmaxf(av, lo), hi);
      a[v] = av;
      d[v] = 1.0f - av;
      float p = 1.0f;  // d^TS by repeated multiplication
#pragma unroll
      for (int i = 0; i < TS; ++i) p *= d[v];
      dts[v] = p;
    }
    if constexpr (kAsync) cp_async_wait<1>();

    // 2. Zero-state scan of the warp's TS tokens -> warp end state.
    {
      float s[VEC];
#pragma unroll
      for (int v = 0; v < VEC; ++v) s[v] = 0.0f;
#pragma unroll
      for (int i = 0; i < TS; ++i) {
        float xv[VEC];
        VecIO<T, VEC>::load(my_x + i * C, xv);
#pragma unroll
        for (int v = 0; v < VEC; ++v) s[v] = a[v] * xv[v] + d[v] * s[v];
      }
#pragma unroll
      for (int v = 0; v < VEC; ++v) s_end[warp][lane * VEC + v] = s[v];
    }
    __syncthreads();

    // 3. Look-back (warp 0).
    if (warp == 0) {
      float agg[VEC], dch[VEC], carry[VEC];
#pragma unroll
      for (int v = 0; v < VEC; ++v) { agg[v] = 0.0f; dch[v] = 1.0f; carry[v] = 0.0f; }
      for (int k = 0; k < WARPS; ++k) {
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          agg[v] = agg[v] * dts[v] + s_end[k][lane * VEC + v];
          dch[v] *= dts[v];
        }
      }
      const int64_t rec = tile * C + lane * VEC;
#pragma unroll
      for (int v = 0; v < VEC; ++v) st_rec(ws.agg + rec + v, agg[v], tag);
      if (chunk == 0) {
        // Carry-in of the first chunk: the caller's initial state (decode
        // continues a sequence) or zero.
        if (init_state != nullptr && lane_active) {
#pragma unroll
          for (int v = 0; v < VEC; ++v) carry[v] = init_state[b * width + c0 + v];
        }
#pragma unroll
        for (int v = 0; v < VEC; ++v) st_rec(ws.incl + rec + v, agg[v] + dch[v] * carry[v], tag);
      } else {
        // Window: aggregates of chunk-1 .. chunk-(LB-1) and, in the farthest
        // slot, the inclusive prefix of chunk-LB; a window that reaches chunk 0
        // reads its inclusive prefix (it holds the initial state's share and is
        // published together with its aggregate).
        const int window = chunk < kLookback ? (int)chunk : kLookback;
        float val[kLookback][VEC];
#pragma unroll
        for (int k = 0; k < kLookback; ++k) {
#pragma unroll
          for (int v = 0; v < VEC; ++v) val[k][v] = 0.0f;
        }
        uint32_t spins = 0;
        for (;;) {
          bool ready = true;
#pragma unroll
          for (int k = 0; k < kLookback; ++k) {
            if (k < window) {
              const int64_t pc = chunk - 1 - k;
              const bool use_incl = k == kLookback - 1 || pc == 0;
              const uint2* src = (use_incl ? ws.incl : ws.agg) + (pc * nseries + series) * C + lane * VEC;
#pragma unroll
              for (int v = 0; v < VEC; ++v) {
                const uint2 r = ld_rec(src + v);
                if (r.y == tag + tag_skew) val[k][v] = __uint_as_float(r.x);
                else ready = false;
              }
            }
          }
          if (__all_sync(0xffffffffu, ready)) break;
          if (++spins > spin_limit) { timed_out = true; break; }
          __nanosleep(20);
        }
        float f[VEC];
#pragma unroll
        for (int v = 0; v < VEC; ++v) f[v] = 1.0f;
#pragma unroll
        for (int k = 0; k < kLookback; ++k) {
#pragma unroll
          for (int v = 0; v < VEC; ++v) {
            carry[v] += f[v] * val[k][v];
            f[v] *= dch[v];
          }
        }
#pragma unroll
        for (int v = 0; v < VEC; ++v) st_rec(ws.incl + rec + v, agg[v] + dch[v] * carry[v], tag);
      }
#pragma unroll
      for (int v = 0; v < VEC; ++v) s_carry[lane * VEC + v] = carry[v];
    }
    __syncthreads();

    // 4. Carry into this warp = tile carry-in pushed through the warps before
    //    it; rescan from it and write y once.
    float s[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) s[v] = s_carry[lane * VEC + v];
    for (int k = 0; k < warp; ++k) {
#pragma unroll
      for (int v = 0; v < VEC; ++v) s[v] = s[v] * dts[v] + s_end[k][lane * VEC + v];
    }
    if (lane_active) {
      T* yrow = y + b * syb + t0 * syn + c0 * syd;
#pragma unroll
      for (int i = 0; i < TS; ++i) {
        float xv[VEC];
        VecIO<T, VEC>::load(my_x + i * C, xv);
#pragma unroll
        for (int v = 0; v < VEC; ++v) s[v] = a[v] * xv[v] + d[v] * s[v];
        if (i < nvalid) VecIO<T, VEC>::store(yrow + i * syn, s);
        if (final_state != nullptr && t0 + i == seq_len - 1) {
#pragma unroll
          for (int v = 0; v < VEC; ++v) final_state[b * width + c0 + v] = s[v];
        }
      }
    }

    cur = nxt;
    nxt += gridDim.x;
    __syncthreads();  // every reader of this slot and of s_end/s_carry is done
    if (nxt < ntiles) stage(nxt, slot);
    if constexpr (kAsync) cp_async_commit();
  }

  if (timed_out && device_status != nullptr) atomicExch(device_status, DWARF_DEVICE_TIMEOUT);
  // The last CTA to exit advances the launch epoch for the next call.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t done = atomicAdd(ws.header + 32, 1u);
    if (done == gridDim.x - 1) {
      ws.header[32] = 0u;
      ws.header[0] = (tag == 0xffffffffu) ? 0u : tag;
      __threadfence();
    }
  }
}

struct EmaPlan {
  int vec, ts, warps;
  int64_t ncb, nseries, nchunks, ntiles;
};

EmaPlan plan_for(int64_t batch, int64_t seq_len, int64_t width, int dtype, bool vector_ok) {
  EmaPlan p{};
  p.vec = dtype == DWARF_F32 ? (vector_ok ? 4 : 1) : (vector_ok ? 8 : 1);
  p.ts = 16;
  p.warps = 4;
  const int64_t C = 32 * p.vec;
  p.ncb = (width + C - 1) / C;
  p.nseries = batch * p.ncb;
  const int64_t CH = (int64_t)p.ts * p.warps;
  p.nchunks = (seq_len + CH - 1) / CH;
  p.ntiles = p.nseries * p.nchunks;
  return p;
}

int64_t workspace_bytes_for(const EmaPlan& p) {
  const int64_t C = 32 * p.vec;
  return kHeaderBytes + 2 * round_up(p.ntiles * C * 8, 256);
}

// Worst case over the two layouts the host may choose for these sizes.
int64_t workspace_bytes_any(int64_t batch, int64_t seq_len, int64_t width, int dtype) {
  int64_t a = workspace_bytes_for(plan_for(batch, seq_len, width, dtype, true));
  int64_t b = workspace_bytes_for(plan_for(batch, seq_len, width, dtype, false));
  return a > b ? a : b;
}

template <typename T, int VEC, int TS, int WARPS, int LB>
int launch_ema_lb(const dwarf_ema_scan_args* a, const EmaPlan& p, cudaStream_t stream) {
  char* base = static_cast<char*>(a->workspace);
  EmaWorkspace ws;
  const int64_t C = 32 * VEC;
  ws.header = reinterpret_cast<uint32_t*>(base);
  ws.agg = reinterpret_cast<uint2*>(base + kHeaderBytes);
  ws.incl = reinterpret_cast<uint2*>(base + kHeaderBytes + round_up(p.ntiles * C * 8, 256));
  const size_t smem = 2 * (size_t)WARPS * TS * C * sizeof(T);
  auto kernel = ema_scan_lookback_kernel<T, VEC, TS, WARPS, LB>;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return DWARF_ERR_LAUNCH;
  int device = 0, sms = kNumSMs, per_sm = 1;
  cudaGetDevice(&device);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, WARPS * 32, smem) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const int64_t grid = std::min<int64_t>(p.ntiles, (int64_t)sms * per_sm);
  const T* x = static_cast<const T*>(a->x);
  T* y = static_cast<T*>(a->y);
  int64_t seq_len = a->seq_len, width = a->width;
  int64_t sxb = a->sxb, sxn = a->sxn, sxd = a->sxd, syb = a->syb, syn = a->syn, syd = a->syd;
  const float* alpha = a->alpha;
  int per_channel = a->alpha_per_channel, clamp = a->clamp;
  float lo = a->floor_, hi = a->ceiling;
  int64_t nseries = p.nseries, ncb = p.ncb, ntiles = p.ntiles;
  int32_t* status = a->device_status;
  const float* init = a->init_state;
  float* fin = a->final_state;
  uint32_t spin_limit = a->wait_limit != 0 ? a->wait_limit : kSpinLimit;
  uint32_t tag_skew = a->test_tag_skew != 0 ? 1u : 0u;
  void* params[] = {&x, &y, &seq_len, &width, &sxb, &sxn, &sxd, &syb, &syn, &syd, &alpha, &per_channel,
                    &clamp, &lo, &hi, &ws, &nseries, &ncb, &ntiles, &status, &init, &fin, &spin_limit, &tag_skew};
  if (cudaLaunchCooperativeKernel((const void*)kernel, dim3((unsigned)grid), dim3(WARPS * 32), params, smem,
                                  stream) != cudaSuccess)
    return DWARF_ERR_LAUNCH;
  return launch_status();
}

template <typename T, int VEC, int TS, int WARPS>
int launch_ema(const dwarf_ema_scan_args* a, const EmaPlan& p, cudaStream_t stream) {
  return p.nseries >= kManySeries ? launch_ema_lb<T, VEC, TS, WARPS, kLookbackMany>(a, p, stream)
                                  : launch_ema_lb<T, VEC, TS, WARPS, kLookbackFew>(a, p, stream);
}


// ---- d alpha: sum over (b, t) of g * (x[t] - y[t-1]), divided by alpha per channel.
// Block = 128 threads across channels (4 each) x kGradGroups row groups of
// kGradRowsPerThread consecutive tokens (kGradRows per block, one batch row);
// y[t-1] is carried from the previous token inside a group, so x, y and g are
// read once plus one y row per group. The groups are summed in shared memory,
// then one atomic per channel (per-channel alpha) or per block (scalar alpha).
__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

constexpr int kGradThreads = 128;
constexpr int kGradGroups = 8;
constexpr int kGradRowsPerThread = 8;
constexpr int kGradRows = kGradGroups * kGradRowsPerThread;

template <typename T>
struct Vec4;
template <>
struct Vec4<float> {
  __device__ static void load(const float* p, float (&o)[4]) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(p));
    o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
  }
};
template <>
struct Vec4<__nv_bfloat16> {
  __device__ static void load(const __nv_bfloat16* p, float (&o)[4]) {
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
    o[0] = __uint_as_float(v.x << 16); o[1] = __uint_as_float(v.x & 0xffff0000u);
    o[2] = __uint_as_float(v.y << 16); o[3] = __uint_as_float(v.y & 0xffff0000u);
  }
};

// VECTOR: 4 consecutive channels per thread read as one 16-B (fp32) or 8-B
// (bf16) load; requires unit channel strides, width % 4 == 0 and aligned rows.
template <typename T, bool VECTOR>
__global__ void __launch_bounds__(kGradThreads * kGradGroups) ema_grad_alpha_kernel(
    const T* __restrict__ x, const T* __restrict__ y, const float* __restrict__ g, int64_t seq_len, int64_t width,
    int64_t sxb, int64_t sxn, int64_t sxd, int64_t syb, int64_t syn, int64_t syd, int64_t sgb, int64_t sgn,
    int64_t sgd, const float* __restrict__ alpha, int per_channel, float* __restrict__ da) {
  constexpr int VEC = 4;
  const int64_t c0 = ((int64_t)blockIdx.x * kGradThreads + threadIdx.x) * VEC;
  const int64_t t0 = (int64_t)blockIdx.y * kGradRows + (int64_t)threadIdx.y * kGradRowsPerThread;
  const int64_t b = blockIdx.z;
  const bool active = c0 < width && t0 < seq_len;
  float acc[VEC];
#pragma unroll
  for (int v = 0; v < VEC; ++v) acc[v] = 0.0f;
  if (active) {
    float prev[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) prev[v] = 0.0f;
    const int64_t t1 = t0 + kGradRowsPerThread < seq_len ? t0 + kGradRowsPerThread : seq_len;
    if constexpr (VECTOR) {
      const T* xp = x + b * sxb + c0;
      const T* yp = y + b * syb + c0;
      const float* gp = g + b * sgb + c0;
      if (t0 > 0) Vec4<T>::load(yp + (t0 - 1) * syn, prev);
#pragma unroll
      for (int i = 0; i < kGradRowsPerThread; ++i) {
        const int64_t t = t0 + i;
        if (t >= t1) break;
        float xv[4], yv[4], gv[4];
        Vec4<T>::load(xp + t * sxn, xv);
        Vec4<T>::load(yp + t * syn, yv);
        Vec4<float>::load(gp + t * sgn, gv);
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          acc[v] = fmaf(gv[v], xv[v] - prev[v], acc[v]);
          prev[v] = yv[v];
        }
      }
    } else {
      if (t0 > 0) {
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          const int64_t c = c0 + v;
          if (c < width) prev[v] = to_f32(y[b * syb + (t0 - 1) * syn + c * syd]);
        }
      }
      for (int64_t t = t0; t < t1; ++t) {
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          const int64_t c = c0 + v;
          if (c < width) {
            const float xv = to_f32(x[b * sxb + t * sxn + c * sxd]);
            const float gv = g[b * sgb + t * sgn + c * sgd];
            acc[v] = fmaf(gv, xv - prev[v], acc[v]);
            prev[v] = to_f32(y[b * syb + t * syn + c * syd]);
          }
        }
      }
    }
  }
  // Sum the row groups: thread (c, 0) ends with the block's partial for its channels.
  __shared__ float red[kGradGroups][kGradThreads * VEC];
#pragma unroll
  for (int v = 0; v < VEC; ++v) red[threadIdx.y][threadIdx.x * VEC + v] = acc[v];
  __syncthreads();
  if (threadIdx.y != 0) return;
#pragma unroll
  for (int v = 0; v < VEC; ++v) {
    float sum = 0.0f;
#pragma unroll
    for (int k = 0; k < kGradGroups; ++k) sum += red[k][threadIdx.x * VEC + v];
    acc[v] = sum;
  }
  if (per_channel) {
    if (c0 < width) {
#pragma unroll
      for (int v = 0; v < VEC; ++v)
        if (c0 + v < width) atomicAdd(da + c0 + v, acc[v] / alpha[c0 + v]);
    }
    return;
  }
  float sum = 0.0f;
#pragma unroll
  for (int v = 0; v < VEC; ++v) sum += acc[v];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  __shared__ float part[kGradThreads / 32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sum;
  asm volatile("bar.sync 1, %0;" ::"n"(kGradThreads));  // the kGradThreads threads of row group 0
  if (threadIdx.x == 0) {
    float total = 0.0f;
#pragma unroll
    for (int w = 0; w < kGradThreads / 32; ++w) total += part[w];
    atomicAdd(da, total / alpha[0]);
  }
}

template <typename T>
int launch_grad_alpha(const dwarf_ema_grad_alpha_args* a, cudaStream_t stream) {
  constexpr int VEC = 4;
  const int64_t cblocks = (a->width + (int64_t)kGradThreads * VEC - 1) / ((int64_t)kGradThreads * VEC);
  const int64_t tblocks = (a->seq_len + kGradRows - 1) / kGradRows;
  if (cblocks > 2147483647LL || tblocks > 65535 || a->batch > 65535) return DWARF_ERR_SHAPE;
  const int64_t ve = 16 / (int64_t)sizeof(T);  // elements per 16 B: x/y rows aligned to 16 B
  const bool vector_ok = a->sxd == 1 && a->syd == 1 && a->sgd == 1 && a->width % VEC == 0 &&
                         aligned16(a->x) && aligned16(a->y) && aligned16(a->g) && a->sxb % ve == 0 &&
                         a->sxn % ve == 0 && a->syb % ve == 0 && a->syn % ve == 0 && a->sgb % 4 == 0 &&
                         a->sgn % 4 == 0;
  dim3 grid((unsigned)cblocks, (unsigned)tblocks, (unsigned)a->batch);
  auto kernel = vector_ok ? ema_grad_alpha_kernel<T, true> : ema_grad_alpha_kernel<T, false>;
  kernel<<<grid, dim3(kGradThreads, kGradGroups), 0, stream>>>(
      static_cast<const T*>(a->x), static_cast<const T*>(a->y), a->g, a->seq_len, a->width, a->sxb, a->sxn,
      a->sxd, a->syb, a->syn, a->syd, a->sgb, a->sgn, a->sgd, a->alpha, a->alpha_per_channel, a->da);
  return launch_status();
}

}  // namespace
}  // namespace dwarf

using namespace dwarf;

extern "C" int64_t dwarf_ema_scan_workspace_bytes(int64_t batch, int64_t seq_len, int64_t width,
                                                  int32_t dtype) {
  if (batch < 0 || seq_len < 0 || width < 0) return -1;
  if (dtype != DWARF_F32 && dtype != DWARF_BF16) return -1;
  return workspace_bytes_any(batch, seq_len, width, dtype);
}

extern "C" int dwarf_ema_scan(const dwarf_ema_scan_args* a, void* stream_) {
  DWARF_CHECK_VERSION(a);
  if (a->dtype != DWARF_F32 && a->dtype != DWARF_BF16) return DWARF_ERR_DTYPE;
  if (a->batch < 0 || a->seq_len < 0 || a->width < 0) return DWARF_ERR_SHAPE;
  if (a->batch == 0 || a->seq_len == 0 || a->width == 0) return DWARF_OK;
  if (!a->x || !a->y || !a->alpha) return DWARF_ERR_NULL;
  if (a->clamp && !(a->floor_ <= a->ceiling)) return DWARF_ERR_VALUE;
  if (a->workspace == nullptr) return DWARF_ERR_WORKSPACE;
  if (!aligned16(a->workspace)) return DWARF_ERR_ALIGN;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const int vec = a->dtype == DWARF_F32 ? 4 : 8;
  const bool vector_ok = a->sxd == 1 && a->syd == 1 && a->width % vec == 0 && a->sxb % vec == 0 &&
                         a->sxn % vec == 0 && a->syb % vec == 0 && a->syn % vec == 0 &&
                         aligned16(a->x) && aligned16(a->y);
  EmaPlan p = plan_for(a->batch, a->seq_len, a->width, a->dtype, vector_ok);
  if (a->workspace_bytes < workspace_bytes_for(p)) return DWARF_ERR_WORKSPACE;
  if (a->dtype == DWARF_F32) {
    return vector_ok ? launch_ema<float, 4, 16, 4>(a, p, stream) : launch_ema<float, 1, 16, 4>(a, p, stream);
  }
  return vector_ok ? launch_ema<__nv_bfloat16, 8, 16, 4>(a, p, stream)
                   : launch_ema<__nv_bfloat16, 1, 16, 4>(a, p, stream);
}

// ---------------------------------------------------------------------------
// Allocation-free variant: the look-back scratch lives in a fixed device array
// owned by the library, for callers that cannot allocate device memory at the
// point of the call. See dwarf_ema_scan_noalloc in include/dwarf_b200.h.

#include <mutex>

namespace {

static __device__ __align__(256) unsigned char g_ema_noalloc_scratch[DWARF_EMA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once
// per device; host code must never use the symbol itself as a pointer).
int scratch_address(void** out) {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) return DWARF_ERR_LAUNCH;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[device] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_ema_noalloc_scratch) != cudaSuccess || ptr == nullptr) return DWARF_ERR_LAUNCH;
    g_scratch_ptr[device] = ptr;
  }
  *out = g_scratch_ptr[device];
  return DWARF_OK;
}

}  // namespace

extern "C" int dwarf_ema_scan_noalloc(const dwarf_ema_scan_args* a, void* stream_) {
  DWARF_CHECK_VERSION(a);
  if (a->dtype != DWARF_F32 && a->dtype != DWARF_BF16) return DWARF_ERR_DTYPE;
  if (a->batch < 0 || a->seq_len < 0 || a->width < 0) return DWARF_ERR_SHAPE;
  if (a->batch == 0 || a->seq_len == 0 || a->width == 0) return DWARF_OK;
  const int64_t need = workspace_bytes_any(a->batch, a->seq_len, a->width, a->dtype);
  if (need > (int64_t)DWARF_EMA_NOALLOC_SCRATCH_BYTES) return DWARF_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  const int st = scratch_address(&scratch);
  if (st != DWARF_OK) return st;
  // Start from a zeroed header and zeroed records, whatever the last call left.
  if (cudaMemsetAsync(scratch, 0, (size_t)need, static_cast<cudaStream_t>(stream_)) != cudaSuccess)
    return DWARF_ERR_LAUNCH;
  dwarf_ema_scan_args local = *a;
  local.workspace = scratch;
  local.workspace_bytes = DWARF_EMA_NOALLOC_SCRATCH_BYTES;
  return dwarf_ema_scan(&local, stream_);
}

extern "C" int dwarf_ema_scan_grad_alpha(const dwarf_ema_grad_alpha_args* a, void* stream_) {
  DWARF_CHECK_VERSION(a);
  if (a->dtype != DWARF_F32 && a->dtype != DWARF_BF16) return DWARF_ERR_DTYPE;
  if (a->batch < 0 || a->seq_len < 0 || a->width < 0) return DWARF_ERR_SHAPE;
  if (!a->da || !a->alpha) return DWARF_ERR_NULL;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const size_t out_bytes = (a->alpha_per_channel ? (size_t)a->width : 1u) * sizeof(float);
  if (cudaMemsetAsync(a->da, 0, out_bytes, stream) != cudaSuccess) return DWARF_ERR_LAUNCH;
  if (a->batch == 0 || a->seq_len == 0 || a->width == 0) return DWARF_OK;
  if (!a->x || !a->y || !a->g) return DWARF_ERR_NULL;
  if (a->dtype == DWARF_F32) return launch_grad_alpha<float>(a, stream);
  return launch_grad_alpha<__nv_bfloat16>(a, stream);
}
