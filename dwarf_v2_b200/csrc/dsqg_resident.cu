// DSQG lattice attention forward with the whole q6 K/V cache of one
// (batch, kv head) resident in shared memory.
//
// Same contract as the gather kernel in dsqg_fwd.cu (it replaces
// _fwd_v22_online, kernels/dsqg_attention_v22.py:698-860, for the q6 cache of
// _DSQGV18GroupedFn.forward, :2197-2352), for the layout the engine itself
// produces: dwarf_q6_pack rows (48 code bytes, contiguous) and fp16 scales
// (contiguous), N % 8 == 0 and small enough for the cache and the tables to
// fit in shared memory (N <= 2176 at the model's 29 offsets; the full
// 96-offset lattice fits at N = 2048).
//
// Why resident: every key row n - off_j is used by the J queries that reach
// it, so the gather kernel reads each row ~J times through L2 and pays an L2
// latency per (query, offset) pair. Here one CTA owns one (b, h): the 100 B
// per row of K+V codes and scales (200 KB at N = 2048) arrive by bulk copies
// (cp.async.bulk, one mbarrier per 256-row chunk, all issued at kernel start)
// and every pair reads its rows from shared memory. A warp's 32 queries read
// 32 consecutive 48-B rows: the 16-B shared loads of each 8-lane phase fall
// on 8 distinct bank groups (conflict-free).
//
// Work split: 512 threads = 16 warps, TWO threads per query (32 head dims and
// two MOVT planes each; the K dot product is completed with one shuffle and
// both threads repeat the per-pair softmax bookkeeping on identical values).
// 122 registers per thread, so 16 warps fit on an SM: at 8 warps (one thread
// per query, 235 registers; still selectable) the kernel stalls on
// fixed-latency dependencies. A round covers 256 queries (one chunk): wait
// for the chunk, flip the sign bit of every 6-bit field in place (two's
// complement -> offset binary, once per row instead of once per pair), then
// each warp walks the offsets in groups of 8: q . bf16(E_j) for its 16
// queries x 8 offsets on tensor cores (mma.sync, through a small per-warp
// transpose buffer into registers), then the group's pairs, one
// online-softmax pass with K and V of a pair consumed together. Offsets that
// reach before token 0 for all of a warp's queries are skipped
// (warp-uniform): at T = 2048 that is ~40% of the (query, offset) grid. The
// running maximum only moves when a score exceeds it by more than 2^8 in the
// exp2 domain, so accumulators are rescaled rarely; weights stay below 2^8.
//
// Decoding without int->float: field i of a 96-bit slice is masked in place
// at bit K_i <= 17 and read as an fp32 denormal, u_i * 2^(K_i - 149), exactly.
// The K dot product pre-scales q_i by 2^(E - K_i) (E per query from max|q|,
// so no product under- or overflows) and the V accumulation pre-scales its
// weight by 2^100; both remove the scaling with one multiply per row. This
// needs fp32 denormals kept (no -ftz), which is the nvcc default.
#include "dsqg_common.cuh"
#include "warp_mma.cuh"

namespace dwarf {
namespace {
using namespace dsqg;
using namespace wmma16;

constexpr int kRQB = 256;  // queries per round == key rows per chunk
constexpr int kRMaxJ = 96;  // the canonical lattice; the shared-memory layout check bounds the rest
constexpr int kRSmemLimit = 232448;  // 227 KB opt-in shared memory per CTA
constexpr float kRescaleLog2 = 8.0f;
constexpr float kVPreScale = 1.2676506002282294e30f;  // 2^100
constexpr int kVPreScaleLog2 = 100;
constexpr int kQeLd = 9;  // row stride (floats) of the per-warp 32 x 8 q.E transpose buffer

struct ResLayout {
  int jp, chunks;
  uint32_t o_kc, o_vc, o_ks, o_vs, o_e, o_qe, o_pb, o_off, o_pbase, o_pgain, o_bar, bytes;
  __host__ __device__ ResLayout(int N, int J, int jl) {
    jp = (J + 7) / 8 * 8;
    chunks = (N + kRQB - 1) / kRQB;
    uint32_t o = 0;
    o_kc = o;    o += (uint32_t)N * 48;
    o_vc = o;    o += (uint32_t)N * 48;
    o_ks = o;    o += (uint32_t)N * 2;
    o_vs = o;    o += (uint32_t)N * 2;
    o_e = o;     o += (uint32_t)jp * 128;
    o_qe = o;    o += (uint32_t)kRQB * kQeLd * 4;
    o_pb = o;    o += (uint32_t)J * 4;
    o_off = o;   o += (uint32_t)J * 4;
    o_pbase = o; o += (uint32_t)jl * 16;
    o_pgain = o; o += (uint32_t)jl * 16;
    o = (o + 7) / 8 * 8;
    o_bar = o;   o += (uint32_t)chunks * 8;
    bytes = o;
  }
};

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// Bounded wait for phase `parity` of an mbarrier; false after kSpinLimit polls.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  for (uint32_t it = 0; it < kSpinLimit; ++it) {
    uint32_t done;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}"
        : "=r"(done) : "r"(bar), "r"(parity) : "memory");
    if (done) return true;
    __nanosleep(64);
  }
  return false;
}
// Global -> shared bulk copy completing on an mbarrier (16-B aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}

__device__ __forceinline__ float den(uint32_t bits) { return __uint_as_float(bits); }

// (a, b) rounded to bf16 and back with one packed conversion.
__device__ __forceinline__ void round_pair_bf16(float& a, float& b) {
  const __nv_bfloat162 t = __floats2bfloat162_rn(a, b);
  const uint32_t w = *reinterpret_cast<const uint32_t*>(&t);
  a = __uint_as_float(w << 16);
  b = __uint_as_float(w & 0xffff0000u);
}

// ex2_approx (common.cuh): arguments here are <= 8; results below 2^-126
// flush to 0, which only drops weights far below the running maximum.

// sum_i q[i] * u_i * 2^(K_i - 149) over the 16 fields of a flipped slice,
// q[i] pre-scaled by 2^(E - K_i): = 2^(E - 149) * sum_i q_i u_i.
__device__ __forceinline__ float dot16(uint32_t w0, uint32_t w1, uint32_t w2, const float* q) {
  const uint32_t w0s = w0 >> 12, w1s = w1 >> 12, w2s = w2 >> 12;
  const uint32_t f5 = __funnelshift_r(w0, w1, 30), f10 = __funnelshift_r(w1, w2, 28);
  float a0 = q[0] * den(w0 & 63u);
  float a1 = q[1] * den(w0 & (63u << 6));
  float a2 = q[2] * den(w0 & (63u << 12));
  float a3 = q[3] * den(w0s & (63u << 6));
  a0 = fmaf(q[4], den(w0s & (63u << 12)), a0);
  a1 = fmaf(q[5], den(f5 & 63u), a1);
  a2 = fmaf(q[6], den(w1 & (63u << 4)), a2);
  a3 = fmaf(q[7], den(w1 & (63u << 10)), a3);
  a0 = fmaf(q[8], den(w1 & (63u << 16)), a0);
  a1 = fmaf(q[9], den(w1s & (63u << 10)), a1);
  a2 = fmaf(q[10], den(f10 & 63u), a2);
  a3 = fmaf(q[11], den(w2 & (63u << 2)), a3);
  a0 = fmaf(q[12], den(w2 & (63u << 8)), a0);
  a1 = fmaf(q[13], den(w2 & (63u << 14)), a1);
  a2 = fmaf(q[14], den(w2s & (63u << 8)), a2);
  a3 = fmaf(q[15], den(w2s & (63u << 14)), a3);
  return (a0 + a1) + (a2 + a3);
}

// acc[i] += wv * u_i * 2^(K_i - 149) over the 16 fields of a flipped slice.
__device__ __forceinline__ void axpy16(uint32_t w0, uint32_t w1, uint32_t w2, float wv, float* acc) {
  const uint32_t w0s = w0 >> 12, w1s = w1 >> 12, w2s = w2 >> 12;
  const uint32_t f5 = __funnelshift_r(w0, w1, 30), f10 = __funnelshift_r(w1, w2, 28);
  acc[0] = fmaf(wv, den(w0 & 63u), acc[0]);
  acc[1] = fmaf(wv, den(w0 & (63u << 6)), acc[1]);
  acc[2] = fmaf(wv, den(w0 & (63u << 12)), acc[2]);
  acc[3] = fmaf(wv, den(w0s & (63u << 6)), acc[3]);
  acc[4] = fmaf(wv, den(w0s & (63u << 12)), acc[4]);
  acc[5] = fmaf(wv, den(f5 & 63u), acc[5]);
  acc[6] = fmaf(wv, den(w1 & (63u << 4)), acc[6]);
  acc[7] = fmaf(wv, den(w1 & (63u << 10)), acc[7]);
  acc[8] = fmaf(wv, den(w1 & (63u << 16)), acc[8]);
  acc[9] = fmaf(wv, den(w1s & (63u << 10)), acc[9]);
  acc[10] = fmaf(wv, den(f10 & 63u), acc[10]);
  acc[11] = fmaf(wv, den(w2 & (63u << 2)), acc[11]);
  acc[12] = fmaf(wv, den(w2 & (63u << 8)), acc[12]);
  acc[13] = fmaf(wv, den(w2 & (63u << 14)), acc[13]);
  acc[14] = fmaf(wv, den(w2s & (63u << 8)), acc[14]);
  acc[15] = fmaf(wv, den(w2s & (63u << 14)), acc[15]);
}

// (a0, a1) += (q0, q1) * (x, y) as one packed fp32x2 FMA (sm_100).
__device__ __forceinline__ void fma2v(float& a0, float& a1, float q0, float q1, float x, float y) {
  asm("{\n.reg .b64 pa, pb, pc;\nmov.b64 pa, {%2, %3};\nmov.b64 pb, {%4, %5};\nmov.b64 pc, {%0, %1};\n"
      "fma.rn.f32x2 pc, pa, pb, pc;\nmov.b64 {%0, %1}, pc;\n}"
      : "+f"(a0), "+f"(a1)
      : "f"(q0), "f"(q1), "f"(x), "f"(y));
}

// dot16 with packed fp32x2 FMAs (two running pairs).
__device__ __forceinline__ float dot16x2(uint32_t w0, uint32_t w1, uint32_t w2, const float* q) {
  const uint32_t w0s = w0 >> 12, w1s = w1 >> 12, w2s = w2 >> 12;
  const uint32_t f5 = __funnelshift_r(w0, w1, 30), f10 = __funnelshift_r(w1, w2, 28);
  float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
  fma2v(a0, a1, q[0], q[1], den(w0 & 63u), den(w0 & (63u << 6)));
  fma2v(b0, b1, q[2], q[3], den(w0 & (63u << 12)), den(w0s & (63u << 6)));
  fma2v(a0, a1, q[4], q[5], den(w0s & (63u << 12)), den(f5 & 63u));
  fma2v(b0, b1, q[6], q[7], den(w1 & (63u << 4)), den(w1 & (63u << 10)));
  fma2v(a0, a1, q[8], q[9], den(w1 & (63u << 16)), den(w1s & (63u << 10)));
  fma2v(b0, b1, q[10], q[11], den(f10 & 63u), den(w2 & (63u << 2)));
  fma2v(a0, a1, q[12], q[13], den(w2 & (63u << 8)), den(w2 & (63u << 14)));
  fma2v(b0, b1, q[14], q[15], den(w2s & (63u << 8)), den(w2s & (63u << 14)));
  return (a0 + a1) + (b0 + b1);
}

// acc[2i], acc[2i+1] += w * (x, y) as one packed fp32x2 FMA (sm_100).
__device__ __forceinline__ void fma2(float& a0, float& a1, float w, float x, float y) {
  asm("{\n.reg .b64 pa, pb, pc;\nmov.b64 pa, {%2, %2};\nmov.b64 pb, {%3, %4};\nmov.b64 pc, {%0, %1};\n"
      "fma.rn.f32x2 pc, pa, pb, pc;\nmov.b64 {%0, %1}, pc;\n}"
      : "+f"(a0), "+f"(a1)
      : "f"(w), "f"(x), "f"(y));
}

// axpy16 with packed fp32x2 FMAs.
__device__ __forceinline__ void axpy16x2(uint32_t w0, uint32_t w1, uint32_t w2, float wv, float* acc) {
  const uint32_t w0s = w0 >> 12, w1s = w1 >> 12, w2s = w2 >> 12;
  const uint32_t f5 = __funnelshift_r(w0, w1, 30), f10 = __funnelshift_r(w1, w2, 28);
  fma2(acc[0], acc[1], wv, den(w0 & 63u), den(w0 & (63u << 6)));
  fma2(acc[2], acc[3], wv, den(w0 & (63u << 12)), den(w0s & (63u << 6)));
  fma2(acc[4], acc[5], wv, den(w0s & (63u << 12)), den(f5 & 63u));
  fma2(acc[6], acc[7], wv, den(w1 & (63u << 4)), den(w1 & (63u << 10)));
  fma2(acc[8], acc[9], wv, den(w1 & (63u << 16)), den(w1s & (63u << 10)));
  fma2(acc[10], acc[11], wv, den(f10 & 63u), den(w2 & (63u << 2)));
  fma2(acc[12], acc[13], wv, den(w2 & (63u << 8)), den(w2 & (63u << 14)));
  fma2(acc[14], acc[15], wv, den(w2s & (63u << 8)), den(w2s & (63u << 14)));
}

// Offset-binary fields rot and rot + 1 of a flipped slice minus the +32 bias.
// PW = (6 * rot) / 32 is the word the pair starts in; off = (6 * rot) % 32.
template <int PW>
__device__ __forceinline__ void movt_pair(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t off, float& a, float& b) {
  uint32_t x;
  if constexpr (PW == 0) x = __funnelshift_r(w0, w1, off);
  else if constexpr (PW == 1) x = __funnelshift_r(w1, w2, off);
  else x = w2 >> off;
  a = __uint_as_float(0x4B000000u | (x & 63u)) - 8388640.0f;          // 2^23 + 32
  b = __uint_as_float(0x4B000000u | ((x >> 6) & 63u)) - 8388640.0f;
}

// TPQ threads per query: 1 (all 64 dims in one thread; 256 threads, 8 warps)
// or 2 (32 dims each, partial dot products combined with one shuffle; 512
// threads, 16 warps). The per-pair score / softmax bookkeeping is repeated in
// both threads of a pair with identical operands, so both hold the same
// running maximum and weights. Two threads per query halve the registers of
// a thread (q and the accumulator are 32 floats each), which doubles the
// warps resident per SM: the kernel is bound by fixed-latency dependencies
// (decode -> FMA chains) at 8 warps per SM.
template <int PW, int TPQ>
__global__ void __launch_bounds__(256 * TPQ, 1) dsqg_resident_kernel(const DsqgParams p, int32_t* status) {
  constexpr int kThreads = 256 * TPQ;
  constexpr int kQW = 32 / TPQ;       // queries per warp
  constexpr int kD = 64 / TPQ;        // head dims per thread
  constexpr int kSL = kD / 16;        // 16-field slices per thread
  constexpr int kW = 3 * kSL;         // 32-bit code words per thread and row
  constexpr int kPL = 4 / TPQ;        // MOVT planes per thread
  constexpr int kMT = kQW / 16;       // m16 tiles of the q.E product per warp
  extern __shared__ __align__(128) unsigned char smem[];
  const int N = (int)p.N, J = p.J, js = p.j_small;
  const ResLayout L(N, J, p.j_large);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int qi = lane / TPQ, hf = lane % TPQ;
  const int64_t h = blockIdx.x, b = blockIdx.y;
  // Query rounds of this CTA: all of them, or one part of a two-way split.
  const int r_begin = gridDim.z == 1 ? 0 : (blockIdx.z == 0 ? p.round_split : 0);
  const int r_end = gridDim.z == 1 ? L.chunks : (blockIdx.z == 0 ? L.chunks : p.round_split);
  const int64_t hk = h / p.kv_group;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + L.o_bar;

  // ---- barriers + all bulk copies (thread 0), tables (everyone)
  if (tid == 0) {
    for (int c = 0; c < L.chunks; ++c) mbar_init(bar0 + 8 * c, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const uint8_t* kc = p.kc + b * p.ccb + hk * p.cch;
    const uint8_t* vc = p.vc + b * p.ccb + hk * p.cch;
    const uint16_t* ks = p.ks + b * p.csb + hk * p.csh;
    const uint16_t* vs = p.vs + b * p.csb + hk * p.csh;
    for (int c = 0; c < r_end; ++c) {  // the key rows this CTA's queries can reach
      const int r0 = c * kRQB;
      const int rows = N - r0 < kRQB ? N - r0 : kRQB;
      const uint32_t bar = bar0 + 8 * c;
      mbar_expect_tx(bar, (uint32_t)rows * 100u);
      bulk_g2s(sbase + L.o_kc + r0 * 48, kc + (int64_t)r0 * 48, rows * 48, bar);
      bulk_g2s(sbase + L.o_vc + r0 * 48, vc + (int64_t)r0 * 48, rows * 48, bar);
      bulk_g2s(sbase + L.o_ks + r0 * 2, ks + r0, rows * 2, bar);
      bulk_g2s(sbase + L.o_vs + r0 * 2, vs + r0, rows * 2, bar);
    }
  }
  const uint32_t e_base = sbase + L.o_e;
  for (int i = tid; i < L.jp * 8; i += kThreads) {
    const int r = i >> 3, c = i & 7;
    uint32_t packed[4] = {0u, 0u, 0u, 0u};
    if (r < J) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float lo = p.se[r * p.sej + (c * 8 + 2 * k) * p.sed];
        const float hi = p.se[r * p.sej + (c * 8 + 2 * k + 1) * p.sed];
        const __nv_bfloat162 two = __floats2bfloat162_rn(lo, hi);
        packed[k] = *reinterpret_cast<const uint32_t*>(&two);
      }
    }
    *reinterpret_cast<uint4*>(smem + (tile_addr(e_base, r, c) - sbase)) =
        make_uint4(packed[0], packed[1], packed[2], packed[3]);
  }
  float* s_pb = reinterpret_cast<float*>(smem + L.o_pb);
  int* s_off = reinterpret_cast<int*>(smem + L.o_off);
  float* s_pbase = reinterpret_cast<float*>(smem + L.o_pbase);
  float* s_pgain = reinterpret_cast<float*>(smem + L.o_pgain);
  for (int j = tid; j < J; j += kThreads) {
    s_pb[j] = p.pos_bias[j * p.spj + h * p.sph] * kLog2e;
    s_off[j] = p.offsets[j];
  }
  for (int i = tid; i < p.j_large * 4; i += kThreads) {
    const int j = i >> 2, r = i & 3;
    s_pbase[i] = p.pbase[j * p.sbj + h * p.sbh + r];
    s_pgain[i] = p.pgain[j * p.sgj + h * p.sgh + r];
  }
  __syncthreads();

  const uint8_t* s_kc = smem + L.o_kc;
  const uint8_t* s_vc = smem + L.o_vc;
  const __half* s_ks = reinterpret_cast<const __half*>(smem + L.o_ks);
  const __half* s_vs = reinterpret_cast<const __half*>(smem + L.o_vs);
  float* qe_buf = reinterpret_cast<float*>(smem + L.o_qe) + warp * kQW * kQeLd;
  const int rot = p.plane_shift;
  const uint32_t rot_off = (uint32_t)(6 * rot) & 31u;
  const float c_score = 0.125f * kLog2e;
  const __nv_bfloat16* qbase = p.q + b * p.sqb + h * p.sqh;
  const float* zbase = p.z + b * p.szb + hk * p.szh + kPL * hf;
  float gain = 1.0f;
  if (p.gain != nullptr)
    gain = p.gain_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.gain)[h])
                       : reinterpret_cast<const float*>(p.gain)[h];

  for (int r = 0; r < r_end; ++r) {
    const int n0 = r * kRQB;
    const bool ok = mbar_wait(bar0 + 8 * r, 0);
    if (__syncthreads_or(!ok)) {
      if (tid == 0) {
        if (status != nullptr) atomicExch(status, DWARF_DEVICE_TIMEOUT);
        // Leave no copy in flight into this CTA's shared memory.
        for (int c = r; c < r_end; ++c) (void)mbar_wait(bar0 + 8 * c, 0);
      }
      return;
    }
    // Two's complement -> offset binary for the chunk's K and V rows.
    {
      const int rows = N - n0 < kRQB ? N - n0 : kRQB;
      uint32_t* kw = reinterpret_cast<uint32_t*>(smem + L.o_kc) + n0 * 12;
      uint32_t* vw = reinterpret_cast<uint32_t*>(smem + L.o_vc) + n0 * 12;
      for (int i = tid; i < rows * 12; i += kThreads) {
        const int k = i % 3;
        const uint32_t m = k == 0 ? 0x20820820u : (k == 1 ? 0x08208208u : 0x82082082u);
        kw[i] ^= m;
        vw[i] ^= m;
      }
    }
    __syncthreads();
    if (r < r_begin) continue;  // block-uniform: an earlier part's rounds (keys staged and flipped only)

    const int wn0 = n0 + warp * kQW;
    if (wn0 >= N) continue;  // warp-uniform; no block barrier follows before the next round

    // ---- per-query state: query n, dims [kD * hf, kD * hf + kD)
    const int n = wn0 + qi;
    const bool row_ok = n < N && n >= p.query_start;
    const int nq = n < N ? n : N - 1;
    float qs[kD];
    float qbias, c1;
    {
      const uint4* src = reinterpret_cast<const uint4*>(qbase + (int64_t)nq * p.sqn + kD * hf);
      float qmax = 0.0f, qsum = 0.0f;
#pragma unroll
      for (int i = 0; i < kD / 8; ++i) {
        const uint4 w = __ldg(src + i);
        const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          qs[8 * i + 2 * k] = __uint_as_float(u[k] << 16);
          qs[8 * i + 2 * k + 1] = __uint_as_float(u[k] & 0xffff0000u);
        }
      }
#pragma unroll
      for (int i = 0; i < kD; ++i) { qmax = fmaxf(qmax, fabsf(qs[i])); qsum += qs[i]; }
      if constexpr (TPQ == 2) {
        qmax = fmaxf(qmax, __shfl_xor_sync(0xffffffffu, qmax, 1));
        qsum += __shfl_xor_sync(0xffffffffu, qsum, 1);
      }
      const int e = (int)((__float_as_uint(qmax) >> 23) & 255u) - 127;  // floor(log2 qmax)
      int E = 125 - e;
      E = E > 100 ? 100 : (E < 22 ? 22 : E);
      // 2^(E - K) for the nine field placements K = 0, 2, ..., 16.
      float sc[9];
#pragma unroll
      for (int k = 0; k < 9; ++k) sc[k] = __int_as_float((127 + E - 2 * k) << 23);
#pragma unroll
      for (int i = 0; i < kD; ++i) qs[i] *= sc[q6_field_shift(i & 15) / 2];
      c1 = __int_as_float((276 - E) << 23);  // 2^(149 - E)
      qbias = -32.0f * qsum;
    }
    // The content-gate row is read only by the epilogue: pull it into L2 now.
    if (p.gate != nullptr && n < N) {
      const __nv_bfloat16* g = p.gate + b * p.sgtb + (int64_t)n * p.sgtn + h * 64 + kD * hf;
      asm volatile("prefetch.global.L2 [%0];" ::"l"(g));
    }
    float gy[kPL];  // y_pre of this query (multiplies phase_gain)
    {
      const float* yrow = p.y + b * p.syb + h * p.syh + (int64_t)nq * p.syn + kPL * hf;
      if constexpr (TPQ == 1) {
        const float4 y4 = *reinterpret_cast<const float4*>(yrow);
        gy[0] = y4.x; gy[1] = y4.y; gy[2] = y4.z; gy[3] = y4.w;
      } else {
        const float2 y2 = *reinterpret_cast<const float2*>(yrow);
        gy[0] = y2.x; gy[1] = y2.y;
      }
    }

    float acc[kD];
#pragma unroll
    for (int i = 0; i < kD; ++i) acc[i] = 0.0f;
    float l = 0.0f, wbias = 0.0f, m = -INFINITY;
    float corr_a[kPL], corr_b[kPL];
#pragma unroll
    for (int pl = 0; pl < kPL; ++pl) { corr_a[pl] = 0.f; corr_b[pl] = 0.f; }

    // Offsets in groups of 8: q . bf16(E_j) for the warp's queries on
    // tensor cores, transposed through qe_buf into this thread's qe[8].
    const int g = lane >> 2, t4 = lane & 3;
    // Offsets whose source row is before token 0 for every query of the
    // warp (off_j > last query) contribute nothing: skip them (warp-uniform).
    const int wlast = wn0 + kQW - 1;
#pragma unroll 1
    for (int j0 = 0; j0 < J; j0 += 8) {
      const int jn = J - j0 < 8 ? J - j0 : 8;
      bool any = false;
      for (int jj = 0; jj < jn; ++jj) any |= s_off[j0 + jj] <= wlast;
      if (!any) continue;
      {
        __syncwarp();
#pragma unroll
        for (int mt = 0; mt < kMT; ++mt) {
          const int ra = min(wn0 + mt * 16 + g, N - 1), rb = min(wn0 + mt * 16 + g + 8, N - 1);
          const __nv_bfloat16* qa = qbase + (int64_t)ra * p.sqn + 2 * t4;
          const __nv_bfloat16* qb2 = qbase + (int64_t)rb * p.sqn + 2 * t4;
          float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint32_t a[4] = {__ldg(reinterpret_cast<const uint32_t*>(qa + ks * 16)),
                                   __ldg(reinterpret_cast<const uint32_t*>(qb2 + ks * 16)),
                                   __ldg(reinterpret_cast<const uint32_t*>(qa + ks * 16 + 8)),
                                   __ldg(reinterpret_cast<const uint32_t*>(qb2 + ks * 16 + 8))};
            uint32_t b0, b1;
            ldsm_x2(tile_addr(e_base, j0 + (lane & 7), ks * 2 + ((lane >> 3) & 1)), b0, b1);
            mma_bf16(c, a, b0, b1);
          }
          float* r0p = qe_buf + (mt * 16 + g) * kQeLd + 2 * t4;
          float* r1p = r0p + 8 * kQeLd;
          r0p[0] = c[0]; r0p[1] = c[1];
          r1p[0] = c[2]; r1p[1] = c[3];
        }
        __syncwarp();
      }
      const float* my_qe = qe_buf + qi * kQeLd;
      // Score of pair (n, j): the K row of the source token from shared memory,
      // q . k in the denormal domain (+ the other thread's half), + q . bf16(E_j),
      // + the position bias. z_pre is loaded for every offset (used by large
      // ones only) so that the function has no branch: two calls in a row form
      // one basic block and their dependency chains interleave.
      auto pair_score = [&](int jj, int& src, bool& valid, float (&zz)[kPL]) -> float {
        const int j = j0 + jj;
        const int s = n - s_off[j];
        valid = row_ok && s >= 0;
        src = valid ? s : 0;
        if constexpr (TPQ == 1) {
          const float4 z4 = __ldg(reinterpret_cast<const float4*>(zbase + (int64_t)src * p.szn));
          zz[0] = z4.x; zz[1] = z4.y; zz[2] = z4.z; zz[3] = z4.w;
        } else {
          const float2 z2 = __ldg(reinterpret_cast<const float2*>(zbase + (int64_t)src * p.szn));
          zz[0] = z2.x; zz[1] = z2.y;
        }
        uint32_t kw[kW];
        if constexpr (TPQ == 1) {
          const uint4* kr = reinterpret_cast<const uint4*>(s_kc + src * 48);
          const uint4 k0 = kr[0], k1 = kr[1], k2 = kr[2];
          kw[0] = k0.x; kw[1] = k0.y; kw[2] = k0.z; kw[3] = k0.w; kw[4] = k1.x; kw[5] = k1.y;
          kw[6] = k1.z; kw[7] = k1.w; kw[8] = k2.x; kw[9] = k2.y; kw[10] = k2.z; kw[11] = k2.w;
        } else {
          const uint2* kr = reinterpret_cast<const uint2*>(s_kc + src * 48 + 24 * hf);
          const uint2 k0 = kr[0], k1 = kr[1], k2 = kr[2];
          kw[0] = k0.x; kw[1] = k0.y; kw[2] = k1.x; kw[3] = k1.y; kw[4] = k2.x; kw[5] = k2.y;
        }
        const float sk = __half2float(s_ks[src]) * (1.0f / 31.0f);
        float P;
        if constexpr (TPQ == 1) {
          P = (dot16x2(kw[0], kw[1], kw[2], qs) + dot16x2(kw[3], kw[4], kw[5], qs + 16)) +
              (dot16x2(kw[6], kw[7], kw[8], qs + 32) + dot16x2(kw[9], kw[10], kw[11], qs + 48));
        } else {
          const float part = dot16x2(kw[0], kw[1], kw[2], qs) + dot16x2(kw[3], kw[4], kw[5], qs + 16);
          const float other = __shfl_xor_sync(0xffffffffu, part, 1);
          P = hf == 0 ? part + other : other + part;  // same sum order in both threads
        }
        const float part = fmaf(P, c1, qbias) * sk;
        const float s2 = fmaf(part + my_qe[jj], c_score, s_pb[j]);
        return valid ? s2 : -INFINITY;
      };
      // Online-softmax update and V accumulation (+ MOVT for large offsets) of one pair.
      // Lazy running maximum: rescale only when a score exceeds it by 2^8.
      auto rescale_to = [&](float smax) {
        if (smax > m + kRescaleLog2) {
          const float f = ex2_approx(m - smax);
#pragma unroll
          for (int i = 0; i < kD; ++i) acc[i] *= f;
          l *= f; wbias *= f;
#pragma unroll
          for (int pl = 0; pl < kPL; ++pl) { corr_a[pl] *= f; corr_b[pl] *= f; }
          m = smax;
        }
      };
      // Weight w of one pair folded into l, the V accumulator and MOVT.
      auto pair_update = [&](int jj, float w, int src, const float (&zz)[kPL]) {
        const int j = j0 + jj;
        const bool large = j >= js;  // warp-uniform
        const float sv = __half2float(s_vs[src]) * (1.0f / 31.0f);
        const float wv = w * sv;
        l += w;
        wbias += wv;
        uint32_t vw[kW];
        if constexpr (TPQ == 1) {
          const uint4* vr = reinterpret_cast<const uint4*>(s_vc + src * 48);
          const uint4 v0 = vr[0], v1 = vr[1], v2 = vr[2];
          vw[0] = v0.x; vw[1] = v0.y; vw[2] = v0.z; vw[3] = v0.w; vw[4] = v1.x; vw[5] = v1.y;
          vw[6] = v1.z; vw[7] = v1.w; vw[8] = v2.x; vw[9] = v2.y; vw[10] = v2.z; vw[11] = v2.w;
        } else {
          const uint2* vr = reinterpret_cast<const uint2*>(s_vc + src * 48 + 24 * hf);
          const uint2 v0 = vr[0], v1 = vr[1], v2 = vr[2];
          vw[0] = v0.x; vw[1] = v0.y; vw[2] = v1.x; vw[3] = v1.y; vw[4] = v2.x; vw[5] = v2.y;
        }
        const float wvs = wv * kVPreScale;
#pragma unroll
        for (int sl = 0; sl < kSL; ++sl) axpy16x2(vw[3 * sl], vw[3 * sl + 1], vw[3 * sl + 2], wvs, acc + 16 * sl);
        if (large) {
          // MOVT: rotate plane r (channels 16 r + rot, + 1) by theta; keep
          // rotated-minus-unrotated so the plain accumulation above stays.
          const int jl = j - js;
#pragma unroll
          for (int pl = 0; pl < kPL; ++pl) {
            const int gp = kPL * hf + pl;  // plane index in the head
            float fa, fb;
            movt_pair<PW>(vw[3 * pl], vw[3 * pl + 1], vw[3 * pl + 2], rot_off, fa, fb);
            const float theta = fmaf(s_pgain[jl * 4 + gp] * gy[pl], zz[pl], s_pbase[jl * 4 + gp]);
            float sn, cs;
            __sincosf(theta, &sn, &cs);
            const float cm1 = cs - 1.0f;
            corr_a[pl] = fmaf(wv, fmaf(cm1, fa, -sn * fb), corr_a[pl]);
            corr_b[pl] = fmaf(wv, fmaf(sn, fa, cm1 * fb), corr_b[pl]);
          }
        }
      };
      // Two pairs per step: both scores first (independent chains), one lazy
      // rescale to the larger, then both weights and the two accumulations.
#pragma unroll 1
      for (int jj = 0; jj < jn; jj += 2) {
        const bool use1 = s_off[j0 + jj] <= wlast;                      // warp-uniform
        const bool use2 = jj + 1 < jn && s_off[j0 + jj + 1] <= wlast;  // warp-uniform
        if (use1 && use2) {
          int src1, src2;
          bool v1, v2;
          float z1[kPL], z2[kPL];
          const float s1 = pair_score(jj, src1, v1, z1);
          const float s2 = pair_score(jj + 1, src2, v2, z2);
          rescale_to(fmaxf(s1, s2));  // one maximum for both: the two weights are independent
          const float w1 = v1 ? ex2_approx(s1 - m) : 0.0f, w2 = v2 ? ex2_approx(s2 - m) : 0.0f;
          pair_update(jj, w1, src1, z1);
          pair_update(jj + 1, w2, src2, z2);
        } else if (use1 || use2) {
          const int jx = use1 ? jj : jj + 1;
          int src;
          bool v;
          float z[kPL];
          const float s = pair_score(jx, src, v, z);
          rescale_to(s);
          pair_update(jx, v ? ex2_approx(s - m) : 0.0f, src, z);
        }
      }
    }

    if (n >= N) continue;
    // ---- epilogue: undo the field scaling and the +32 bias, add MOVT
    // corrections, normalise, optional gain / gate, bf16 store.
    const float bias = 32.0f * wbias;
    const float inv_l = l > 0.0f ? 1.0f / l : 0.0f;
    __nv_bfloat16* orow = p.out + b * p.sob + h * p.soh + (int64_t)n * p.son + kD * hf;
    const __nv_bfloat16* grow =
        p.gate != nullptr ? p.gate + b * p.sgtb + (int64_t)n * p.sgtn + h * 64 + kD * hf : nullptr;
#pragma unroll
    for (int sl = 0; sl < kSL; ++sl) {
      float o[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float v = fmaf(acc[16 * sl + i], __int_as_float((127 + 149 - kVPreScaleLog2 - q6_field_shift(i)) << 23),
                       -bias);
        if (i == rot) v += corr_a[sl];
        if (i == rot + 1) v += corr_b[sl];
        o[i] = v * inv_l;
      }
#pragma unroll
      for (int i = 0; i < 16; i += 2) round_pair_bf16(o[i], o[i + 1]);
      if (p.gain != nullptr) {
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] *= gain;
        if (p.gain_bf16) {
#pragma unroll
          for (int i = 0; i < 16; i += 2) round_pair_bf16(o[i], o[i + 1]);
        }
      }
      if (grow != nullptr) {
        const uint4* gp = reinterpret_cast<const uint4*>(grow + 16 * sl);
        const uint4 gw[2] = {__ldg(gp), __ldg(gp + 1)};
        float gv[16];
        bf16x16_to_f32(gw, gv);
        // sigmoid(gate) rounded to bf16 (the reference's bf16 sigmoid) from the
        // hardware exp2 and reciprocal: their few-ulp fp32 error is absorbed by the
        // bf16 rounding except at rounding ties.
        const bool round_out = p.gain_bf16 || p.gain == nullptr;
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          float s0 = __fdividef(1.0f, 1.0f + __expf(-gv[i])), s1 = __fdividef(1.0f, 1.0f + __expf(-gv[i + 1]));
          round_pair_bf16(s0, s1);
          float o0 = o[i] * s0, o1 = o[i + 1] * s1;
          if (round_out) round_pair_bf16(o0, o1);
          o[i] = o0;
          o[i + 1] = o1;
        }
      }
      uint4 packed[2];
      uint32_t* pw = reinterpret_cast<uint32_t*>(packed);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const __nv_bfloat162 two = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
        pw[i] = *reinterpret_cast<const uint32_t*>(&two);
      }
      uint4* dst = reinterpret_cast<uint4*>(orow + 16 * sl);
      dst[0] = packed[0];
      dst[1] = packed[1];
    }
    if (p.lse != nullptr && hf == 0)
      p.lse[b * p.slb + h * p.slh + (int64_t)n * p.sln] = l > 0.0f ? m * 0.6931471805599453f + logf(l) : -INFINITY;
  }
}

bool al(const void* ptr, uintptr_t a) { return (reinterpret_cast<uintptr_t>(ptr) & (a - 1)) == 0; }

}  // namespace

int dsqg_resident_launch(const DsqgParams& p, int64_t B, cudaStream_t stream) {
  // Layout and size limits of the resident kernel; anything else goes to the gather kernel.
  if (p.kc == nullptr || p.J > kRMaxJ || p.N % 8 != 0 || p.cct != 48 || p.cst != 1) return kNotApplicable;
  if (!al(p.kc, 16) || !al(p.vc, 16) || !al(p.ks, 16) || !al(p.vs, 16) || p.ccb % 16 || p.cch % 16 ||
      (p.csb * 2) % 16 || (p.csh * 2) % 16)
    return kNotApplicable;
  if (!al(p.y, 16) || !al(p.z, 16) || p.syb % 4 || p.syh % 4 || p.syn % 4 || p.szb % 4 || p.szh % 4 || p.szn % 4)
    return kNotApplicable;
  if (p.gate != nullptr && p.sgtn % 8) return kNotApplicable;
  const ResLayout L((int)p.N, p.J, p.j_large);
  if (p.N > 4096 || L.bytes > (uint32_t)kRSmemLimit || B > 65535 || p.H > 65535) return kNotApplicable;
  const int pw = (6 * p.plane_shift) >> 5;
  // Threads per query: 2 by default; DWARF_DSQG_RES_TPQ=1 selects one thread per query.
  static const int tpq = [] {
    const char* e = getenv("DWARF_DSQG_RES_TPQ");
    return (e && e[0] == '1') ? 1 : 2;
  }();
  using KernelFn = void (*)(const DsqgParams, int32_t*);
  KernelFn kernel;
  if (tpq == 1)
    kernel = pw == 0 ? dsqg_resident_kernel<0, 1> : (pw == 1 ? dsqg_resident_kernel<1, 1> : dsqg_resident_kernel<2, 1>);
  else
    kernel = pw == 0 ? dsqg_resident_kernel<0, 2> : (pw == 1 ? dsqg_resident_kernel<1, 2> : dsqg_resident_kernel<2, 2>);
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.bytes) != cudaSuccess)
    return DWARF_ERR_LAUNCH;
  // Two-way split of each (b, h) by query rounds when the (b, h) count would leave
  // the last wave short (fewer than four waves): the later rounds (more offsets in
  // reach, ~3/4 of the work) as one CTA, dispatched first, the earlier ones as
  // another, so the short CTAs fill the last wave. DWARF_DSQG_SPLIT=1 / 2 forces
  // one part / two parts (read on every call).
  int sms = kNumSMs, device = 0;
  if (cudaGetDevice(&device) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  const char* force = getenv("DWARF_DSQG_SPLIT");
  bool split = L.chunks >= 4 && B * p.H < 4LL * sms;
  if (force != nullptr && force[0] == '1') split = false;
  if (force != nullptr && force[0] == '2') split = L.chunks >= 2;
  DsqgParams pr = p;
  pr.round_split = split ? (L.chunks * 3 + 4) / 8 : 0;
  if (split && pr.round_split < 1) pr.round_split = 1;
  dim3 grid((unsigned)p.H, (unsigned)B, split ? 2u : 1u);
  kernel<<<grid, 256 * tpq, L.bytes, stream>>>(pr, p.status);
  return launch_status();
}

}  // namespace dwarf
