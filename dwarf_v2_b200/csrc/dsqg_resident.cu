// DSQG lattice attention forward with the whole q6 K/V cache of one
// (batch, kv head) resident in shared memory.
//
// Same contract as the gather kernel in dsqg_fwd.cu (it replaces
// _fwd_v22_online, kernels/dsqg_attention_v22.py:698-860, for the q6 cache of
// _DSQGV18GroupedFn.forward, :2197-2352), for the layout the engine itself
// produces: dwarf_q6_pack rows (48 code bytes, contiguous) and fp16 scales
// (contiguous), N <= 2048 with N % 8 == 0, J <= 32.
//
// Why resident: every key row n - off_j is used by the J queries that reach
// it, so the gather kernel reads each row ~J times through L2 and pays an L2
// latency per (query, offset) pair. Here one CTA owns one (b, h): the 100 B
// per row of K+V codes and scales (200 KB at N = 2048) arrive by bulk copies
// (cp.async.bulk, one mbarrier per 192-row chunk, all issued at kernel start)
// and every pair reads its row from shared memory. Rows of consecutive
// queries are consecutive 48-B rows, which keeps the 64-bit shared loads of a
// half-warp on 16 distinct bank pairs (conflict-free).
//
// Work split: 384 threads = 12 warps; a round covers 192 queries (one chunk),
// 2 threads per query (32 head dims each). Per round: wait for the round's
// chunk, flip the sign bit of every 6-bit field in place (two's complement
// -> offset binary, once per row instead of once per pair), then each warp
// computes q . bf16(E_j) for its 16 queries on tensor cores (mma.sync) and
// runs one online-softmax pass over the offsets with K and V of a pair
// consumed together. The running maximum is only moved when a score exceeds
// it by more than 2^8 in the exp2 domain, so accumulators are rescaled
// rarely; weights stay below 2^8.
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

constexpr int kRThreads = 384;
constexpr int kRQB = 192;  // queries per round == key rows per chunk
constexpr int kRMaxJ = 32;
constexpr int kRSmemLimit = 232448;  // 227 KB opt-in shared memory per CTA
constexpr float kRescaleLog2 = 8.0f;
constexpr float kVPreScale = 1.2676506002282294e30f;  // 2^100
constexpr int kVPreScaleLog2 = 100;

struct ResLayout {
  int jp, qe_ld, chunks;
  uint32_t o_kc, o_vc, o_ks, o_vs, o_e, o_qe, o_pb, o_off, o_pbase, o_pgain, o_bar, bytes;
  __host__ __device__ ResLayout(int N, int J, int jl) {
    jp = (J + 7) / 8 * 8;
    qe_ld = J | 1;  // odd row stride: the 16 rows a warp reads sit in 16 banks
    chunks = (N + kRQB - 1) / kRQB;
    uint32_t o = 0;
    o_kc = o;    o += (uint32_t)N * 48;
    o_vc = o;    o += (uint32_t)N * 48;
    o_ks = o;    o += (uint32_t)N * 2;
    o_vs = o;    o += (uint32_t)N * 2;
    o_e = o;     o += (uint32_t)jp * 128;
    o_qe = o;    o += (uint32_t)kRQB * qe_ld * 4;
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

struct RState {
  float acc[32];
  float l, wbias, m;
  float corr_a[2], corr_b[2];
};

template <int PW>
__global__ void __launch_bounds__(kRThreads, 1) dsqg_resident_kernel(const DsqgParams p, int32_t* status) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int N = (int)p.N, J = p.J, js = p.j_small;
  const ResLayout L(N, J, p.j_large);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t h = blockIdx.x, b = blockIdx.y;
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
    for (int c = 0; c < L.chunks; ++c) {
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
  for (int i = tid; i < L.jp * 8; i += kRThreads) {
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
  for (int j = tid; j < J; j += kRThreads) {
    s_pb[j] = p.pos_bias[j * p.spj + h * p.sph] * kLog2e;
    s_off[j] = p.offsets[j];
  }
  for (int i = tid; i < p.j_large * 4; i += kRThreads) {
    const int j = i >> 2, r = i & 3;
    s_pbase[i] = p.pbase[j * p.sbj + h * p.sbh + r];
    s_pgain[i] = p.pgain[j * p.sgj + h * p.sgh + r];
  }
  __syncthreads();

  const uint8_t* s_kc = smem + L.o_kc;
  const uint8_t* s_vc = smem + L.o_vc;
  const __half* s_ks = reinterpret_cast<const __half*>(smem + L.o_ks);
  const __half* s_vs = reinterpret_cast<const __half*>(smem + L.o_vs);
  float* s_qe = reinterpret_cast<float*>(smem + L.o_qe);
  const int sub = lane & 1;
  const int rot = p.plane_shift;
  const uint32_t rot_off = (uint32_t)(6 * rot) & 31u;
  const float c_score = 0.125f * kLog2e;
  const __nv_bfloat16* qbase = p.q + b * p.sqb + h * p.sqh;
  const float* zbase = p.z + b * p.szb + hk * p.szh + sub * 2;
  float gain = 1.0f;
  if (p.gain != nullptr)
    gain = p.gain_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.gain)[h])
                       : reinterpret_cast<const float*>(p.gain)[h];

  for (int r = 0; r < L.chunks; ++r) {
    const int n0 = r * kRQB;
    const bool ok = mbar_wait(bar0 + 8 * r, 0);
    if (__syncthreads_or(!ok)) {
      if (tid == 0) {
        if (status != nullptr) atomicExch(status, DWARF_DEVICE_TIMEOUT);
        // Leave no copy in flight into this CTA's shared memory.
        for (int c = r; c < L.chunks; ++c) (void)mbar_wait(bar0 + 8 * c, 0);
      }
      return;
    }
    // Two's complement -> offset binary for the chunk's K and V rows.
    {
      const int rows = N - n0 < kRQB ? N - n0 : kRQB;
      uint32_t* kw = reinterpret_cast<uint32_t*>(smem + L.o_kc) + n0 * 12;
      uint32_t* vw = reinterpret_cast<uint32_t*>(smem + L.o_vc) + n0 * 12;
      for (int i = tid; i < rows * 12; i += kRThreads) {
        const int k = i % 3;
        const uint32_t m = k == 0 ? 0x20820820u : (k == 1 ? 0x08208208u : 0x82082082u);
        kw[i] ^= m;
        vw[i] ^= m;
      }
    }
    __syncthreads();

    const int wn0 = n0 + warp * 16;
    if (wn0 >= N) continue;  // warp-uniform; no block barrier follows before the next round

    // ---- q . bf16(E_j) for this warp's 16 queries (mma m16n8k16, A straight from global)
    float* qe_w = s_qe + warp * 16 * L.qe_ld;
    {
      const int g = lane >> 2, t4 = lane & 3;
      const int ra = wn0 + g < N ? wn0 + g : N - 1;
      const int rb = wn0 + g + 8 < N ? wn0 + g + 8 : N - 1;
      const __nv_bfloat16* qa = qbase + (int64_t)ra * p.sqn + 2 * t4;
      const __nv_bfloat16* qb2 = qbase + (int64_t)rb * p.sqn + 2 * t4;
      uint32_t a[4][4];
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        a[ks][0] = __ldg(reinterpret_cast<const uint32_t*>(qa + ks * 16));
        a[ks][1] = __ldg(reinterpret_cast<const uint32_t*>(qb2 + ks * 16));
        a[ks][2] = __ldg(reinterpret_cast<const uint32_t*>(qa + ks * 16 + 8));
        a[ks][3] = __ldg(reinterpret_cast<const uint32_t*>(qb2 + ks * 16 + 8));
      }
      for (int nt = 0; nt < L.jp / 8; ++nt) {
        float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          uint32_t b0, b1;
          ldsm_x2(tile_addr(e_base, nt * 8 + (lane & 7), ks * 2 + ((lane >> 3) & 1)), b0, b1);
          mma_bf16(c, a[ks], b0, b1);
        }
        const int col = nt * 8 + 2 * t4;
        if (col < J) { qe_w[g * L.qe_ld + col] = c[0]; qe_w[(g + 8) * L.qe_ld + col] = c[2]; }
        if (col + 1 < J) { qe_w[g * L.qe_ld + col + 1] = c[1]; qe_w[(g + 8) * L.qe_ld + col + 1] = c[3]; }
      }
    }
    __syncwarp();

    // ---- per-query state (2 threads per query, 32 dims each)
    const int qi = lane >> 1;
    const int n = wn0 + qi;
    const bool row_ok = n < N && n >= p.query_start;
    const int nq = n < N ? n : N - 1;
    const float* my_qe = qe_w + qi * L.qe_ld;
    float qs[32];
    float qbias, c1;
    {
      const uint4* src = reinterpret_cast<const uint4*>(qbase + (int64_t)nq * p.sqn + sub * 32);
      uint4 w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) w[i] = __ldg(src + i);
      float qmax = 0.0f, qsum = 0.0f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t u[4] = {w[i].x, w[i].y, w[i].z, w[i].w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          qs[8 * i + 2 * k] = __uint_as_float(u[k] << 16);
          qs[8 * i + 2 * k + 1] = __uint_as_float(u[k] & 0xffff0000u);
        }
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) { qmax = fmaxf(qmax, fabsf(qs[i])); qsum += qs[i]; }
      qmax = fmaxf(qmax, __shfl_xor_sync(0xffffffffu, qmax, 1));
      const int e = (int)((__float_as_uint(qmax) >> 23) & 255u) - 127;  // floor(log2 qmax)
      int E = 125 - e;
      E = E > 100 ? 100 : (E < 22 ? 22 : E);
#pragma unroll
      for (int i = 0; i < 32; ++i) qs[i] *= __int_as_float((127 + E - q6_field_shift(i & 15)) << 23);
      c1 = __int_as_float((276 - E) << 23);  // 2^(149 - E)
      qbias = -32.0f * qsum;
    }
    float yq[2];
    {
      const float2 y2 = *reinterpret_cast<const float2*>(p.y + b * p.syb + h * p.syh + (int64_t)nq * p.syn + sub * 2);
      yq[0] = y2.x; yq[1] = y2.y;
    }

    RState st;
#pragma unroll
    for (int i = 0; i < 32; ++i) st.acc[i] = 0.0f;
    st.l = 0.0f; st.wbias = 0.0f; st.m = -INFINITY;
    st.corr_a[0] = st.corr_a[1] = st.corr_b[0] = st.corr_b[1] = 0.0f;

    // One (query, offset) pair; returns the weight-times-step of the pair.
    auto pair = [&](int j, bool valid, int src) -> float {
      const uint32_t* kr = reinterpret_cast<const uint32_t*>(s_kc + src * 48 + sub * 24);
      const uint2 k01 = *reinterpret_cast<const uint2*>(kr);
      const uint2 k23 = *reinterpret_cast<const uint2*>(kr + 2);
      const uint2 k45 = *reinterpret_cast<const uint2*>(kr + 4);
      const float sk = __half2float(s_ks[src]) * (1.0f / 31.0f);
      const float P = dot16(k01.x, k01.y, k23.x, qs) + dot16(k23.y, k45.x, k45.y, qs + 16);
      float part = fmaf(P, c1, qbias) * sk;
      part += __shfl_xor_sync(0xffffffffu, part, 1);
      float s2 = fmaf(part + my_qe[j], c_score, s_pb[j]);
      s2 = valid ? s2 : -INFINITY;
      if (s2 > st.m + kRescaleLog2) {  // uniform within the query's two threads
        const float f = exp2f(st.m - s2);
#pragma unroll
        for (int i = 0; i < 32; ++i) st.acc[i] *= f;
        st.l *= f; st.wbias *= f;
        st.corr_a[0] *= f; st.corr_a[1] *= f; st.corr_b[0] *= f; st.corr_b[1] *= f;
        st.m = s2;
      }
      const float w = valid ? exp2f(s2 - st.m) : 0.0f;
      const float sv = __half2float(s_vs[src]) * (1.0f / 31.0f);
      const float wv = w * sv;
      st.l += w;
      st.wbias += wv;
      const uint32_t* vr = reinterpret_cast<const uint32_t*>(s_vc + src * 48 + sub * 24);
      const uint2 v01 = *reinterpret_cast<const uint2*>(vr);
      const uint2 v23 = *reinterpret_cast<const uint2*>(vr + 2);
      const uint2 v45 = *reinterpret_cast<const uint2*>(vr + 4);
      const float wvs = wv * kVPreScale;
      axpy16(v01.x, v01.y, v23.x, wvs, st.acc);
      axpy16(v23.y, v45.x, v45.y, wvs, st.acc + 16);
      return wv;
    };

    // Small band: no MOVT.
    for (int j = 0; j < js; ++j) {
      const int s = n - s_off[j];
      const bool valid = row_ok && s >= 0;
      (void)pair(j, valid, valid ? s : 0);
    }
    // Large band: MOVT plane rotation of the two planes this thread owns.
    {
      float2 zn = make_float2(0.f, 0.f);
      if (js < J) {
        const int s = nq - s_off[js];  // nq: rows past N must not index past the z rows
        zn = *reinterpret_cast<const float2*>(zbase + (int64_t)(s >= 0 ? s : 0) * p.szn);
      }
      for (int j = js; j < J; ++j) {
        const int s = n - s_off[j];
        const bool valid = row_ok && s >= 0;
        const int src = valid ? s : 0;
        const float2 zc = zn;
        if (j + 1 < J) {
          const int s1 = nq - s_off[j + 1];
          zn = *reinterpret_cast<const float2*>(zbase + (int64_t)(s1 >= 0 ? s1 : 0) * p.szn);
        }
        const float wv = pair(j, valid, src);
        const uint32_t* vr = reinterpret_cast<const uint32_t*>(s_vc + src * 48 + sub * 24);
        const int jl = j - js;
        const float zz[2] = {zc.x, zc.y};
#pragma unroll
        for (int sl = 0; sl < 2; ++sl) {
          const uint32_t w0 = vr[3 * sl], w1 = vr[3 * sl + 1], w2 = vr[3 * sl + 2];
          float fa, fb;
          movt_pair<PW>(w0, w1, w2, rot_off, fa, fb);
          const int plane = sub * 2 + sl;
          const float theta = fmaf(s_pgain[jl * 4 + plane] * yq[sl], zz[sl], s_pbase[jl * 4 + plane]);
          float sn, cs;
          __sincosf(theta, &sn, &cs);
          const float cm1 = cs - 1.0f;
          st.corr_a[sl] = fmaf(wv, fmaf(cm1, fa, -sn * fb), st.corr_a[sl]);
          st.corr_b[sl] = fmaf(wv, fmaf(sn, fa, cm1 * fb), st.corr_b[sl]);
        }
      }
    }

    if (n >= N) continue;
    // ---- epilogue: undo the field scaling and the +32 bias, add MOVT
    // corrections, normalise, optional gain / gate, bf16 store.
    const float bias = 32.0f * st.wbias;
    const int d0 = sub * 32;
#pragma unroll
    for (int sl = 0; sl < 2; ++sl) {
      float o[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float v = fmaf(st.acc[16 * sl + i], __int_as_float((127 + 149 - kVPreScaleLog2 - q6_field_shift(i)) << 23),
                       -bias);
        if (i == rot) v += st.corr_a[sl];
        if (i == rot + 1) v += st.corr_b[sl];
        o[i] = st.l > 0.0f ? round_bf16(v / st.l) : 0.0f;
      }
      if (p.gain != nullptr) {
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] = p.gain_bf16 ? round_bf16(o[i] * gain) : o[i] * gain;
      }
      if (p.gate != nullptr) {
        const uint4* gp = reinterpret_cast<const uint4*>(p.gate + b * p.sgtb + (int64_t)n * p.sgtn + h * 64 + d0 + 16 * sl);
        const uint4 gw[2] = {__ldg(gp), __ldg(gp + 1)};
        float gv[16];
        bf16x16_to_f32(gw, gv);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float sg = round_bf16(1.0f / (1.0f + expf(-gv[i])));
          o[i] = p.gain_bf16 || p.gain == nullptr ? round_bf16(o[i] * sg) : o[i] * sg;
        }
      }
      uint4 packed[2];
      uint32_t* pw = reinterpret_cast<uint32_t*>(packed);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const __nv_bfloat162 two = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
        pw[i] = *reinterpret_cast<const uint32_t*>(&two);
      }
      uint4* dst = reinterpret_cast<uint4*>(p.out + b * p.sob + h * p.soh + (int64_t)n * p.son + d0 + 16 * sl);
      dst[0] = packed[0];
      dst[1] = packed[1];
    }
    if (p.lse != nullptr && sub == 0)
      p.lse[b * p.slb + h * p.slh + (int64_t)n * p.sln] =
          st.l > 0.0f ? st.m * 0.6931471805599453f + logf(st.l) : -INFINITY;
  }
}

bool al(const void* ptr, uintptr_t a) { return (reinterpret_cast<uintptr_t>(ptr) & (a - 1)) == 0; }

}  // namespace

int dsqg_resident_launch(const DsqgParams& p, int64_t B, cudaStream_t stream) {
  // Layout and size limits of the resident kernel; anything else goes to the gather kernel.
  if (p.kc == nullptr || p.J > kRMaxJ || p.N > 2048 || p.N % 8 != 0 || p.cct != 48 || p.cst != 1) return kNotApplicable;
  if (!al(p.kc, 16) || !al(p.vc, 16) || !al(p.ks, 16) || !al(p.vs, 16) || p.ccb % 16 || p.cch % 16 ||
      (p.csb * 2) % 16 || (p.csh * 2) % 16)
    return kNotApplicable;
  if (!al(p.y, 8) || !al(p.z, 8) || p.syb % 2 || p.syh % 2 || p.syn % 2 || p.szb % 2 || p.szh % 2 || p.szn % 2)
    return kNotApplicable;
  if (p.gate != nullptr && p.sgtn % 8) return kNotApplicable;
  const ResLayout L((int)p.N, p.J, p.j_large);
  if (L.bytes > (uint32_t)kRSmemLimit || B > 65535 || p.H > 0x7fffffff) return kNotApplicable;
  const int pw = (6 * p.plane_shift) >> 5;
  auto kernel = pw == 0 ? dsqg_resident_kernel<0> : (pw == 1 ? dsqg_resident_kernel<1> : dsqg_resident_kernel<2>);
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.bytes) != cudaSuccess)
    return DWARF_ERR_LAUNCH;
  dim3 grid((unsigned)p.H, (unsigned)B);
  kernel<<<grid, kRThreads, L.bytes, stream>>>(p, p.status);
  return launch_status();
}

}  // namespace dwarf
