// DSQG lattice attention forward (CUDA cores, fp32 math).
//
// Replaces _fwd_v22_online (kernels/dsqg_attention_v22.py:698-860), launched
// by _DSQGV18GroupedFn.forward (:2197-2352). Same semantics, same order of
// offsets, same online softmax in the exp2 domain and the same bf16 rounding
// of the scale-embedding "virtual key" (:760-763); differences to the
// reference are fp32 summation order only.
//
// Mapping: one CTA = 64 consecutive queries of one (batch, head); 4 threads
// per query, each owning 16 of the 64 head dims (32 B of a bf16 row, or 12 B
// of a q6 row). A query's dot product is reduced over its 4 threads with two
// xor-shuffles. MOVT plane r (channels 16r+shift, 16r+shift+1) lies inside the
// slice of thread r, so each thread rotates exactly one plane. K/V rows are
// gathered straight from global memory (rows of neighbouring queries are
// neighbouring rows, so each warp reads 8 whole rows per offset), with the
// next offset's row prefetched while the current one is consumed.
// The scale-embedding term q . bf16(E_j) of every (query, offset) is one
// 64 x J x 64 bf16 tensor-core product per CTA (mma.sync), so the per-pair
// loop only handles q . k. Scores are computed in a first pass and the V
// accumulation runs in a second pass against the final maximum, which removes
// the per-offset accumulator rescaling of the online form.
#include "common.cuh"
#include "q6_format.cuh"
#include "warp_mma.cuh"
#include "dsqg_common.cuh"

#include <cstdlib>
#include <type_traits>

namespace dwarf {
namespace {
using namespace dsqg;

constexpr int kThreads = 256;  // threads per CTA

// Unscaled u of code i (runtime index) -- used for the two MOVT plane channels.
__device__ __forceinline__ float q6_u_at(const uint32_t (&w)[3], int i) {
  const int bit = 6 * i, word = bit >> 5, off = bit & 31;
  const uint32_t lo = word == 0 ? w[0] : (word == 1 ? w[1] : w[2]);
  const uint32_t hi = word == 0 ? w[1] : w[2];
  return (float)(__funnelshift_r(lo, hi, off) & 63u);
}

// One gathered row slice: bf16 (2 x uint4) or q6 (3 x u32 + fp16 scale).
template <bool Q6>
struct RowSlice;
template <>
struct RowSlice<false> {
  uint4 w[2];
  __device__ __forceinline__ void load(const __nv_bfloat16* base, bool ok) {
    if (ok) {
      const uint4* p = reinterpret_cast<const uint4*>(base);
      w[0] = __ldg(p);
      w[1] = __ldg(p + 1);
    } else {
      w[0] = w[1] = make_uint4(0, 0, 0, 0);
    }
  }
  __device__ __forceinline__ void to_f32(float (&o)[16]) const { bf16x16_to_f32(w, o); }
};
template <>
struct RowSlice<true> {
  uint32_t w[3];
  uint16_t s;
  __device__ __forceinline__ void load(const uint8_t* codes, const uint16_t* scale, bool ok) {
    if (ok) {
      const uint32_t* p = reinterpret_cast<const uint32_t*>(codes);
      w[0] = __ldg(p);
      w[1] = __ldg(p + 1);
      w[2] = __ldg(p + 2);
      s = __ldg(scale);
    } else {
      w[0] = w[1] = w[2] = 0u;
      s = 0;
    }
  }
  // Offset-binary values u_d * 2^K_d (see q6_scaled16), the flipped words
  // and the dequantisation step.
  __device__ __forceinline__ void to_scaled(float (&o)[16], uint32_t (&t)[3], float& step) const {
    t[0] = w[0]; t[1] = w[1]; t[2] = w[2];
    q6_flip_sign_bits(t);
    q6_scaled16(t, o);
    // float(s) / 31 up to one rounding (a reciprocal multiply instead of an
    // IEEE division per gathered row; the attention tolerance absorbs it).
    step = __half2float(__ushort_as_half(s)) * (1.0f / 31.0f);
  }
};

// Shared-memory carve-up of one CTA (QB queries of one (b, h)).
struct DsqgSmem {
  int jp;       // J rounded up to a multiple of 8 (mma n-tiles)
  int qe_ld;    // row stride of qe (jp + 1 floats)
  int sc_ld;    // row stride of sc (J + 1 floats)
  size_t bytes;
  size_t o_q, o_e, o_qe, o_sc, o_pb, o_off, o_pbase, o_pgain;
  __host__ __device__ DsqgSmem(int J, int j_large, int qb) {
    jp = (J + 7) / 8 * 8;
    qe_ld = jp + 1;
    sc_ld = J + 1;
    size_t o = 0;
    o_q = o;      o += (size_t)qb * 128;                // bf16 Q tile, swizzled
    o_e = o;      o += (size_t)jp * 128;                // bf16(scale_embed), swizzled
    o_qe = o;     o += (size_t)qb * qe_ld * 4;          // q . bf16(E_j) (fp32)
    o_sc = o;     o += (size_t)qb * sc_ld * 4;          // scores of pass 1
    o_pb = o;     o += (size_t)J * 4;
    o_off = o;    o += (size_t)J * 4;
    o_pbase = o;  o += (size_t)j_large * 16;
    o_pgain = o;  o += (size_t)j_large * 16;
    bytes = (o + 15) / 16 * 16;
  }
};

// Two passes per query: (1) scores of every live offset from K rows plus the
// tensor-core q.E term, running max; (2) exp2 weights against the final max
// and the V accumulation (no accumulator rescaling), MOVT planes rotated in
// the owning thread. TPQ threads share a query, each owning 64/TPQ dims and
// 4/TPQ MOVT planes; a CTA of 256 threads covers QB = 256/TPQ queries.
template <bool Q6, int TPQ>
__global__ void __launch_bounds__(kThreads)
dsqg_fwd_kernel(const DsqgParams p) {
  using namespace wmma16;
  constexpr int QB = kThreads / TPQ;       // queries per CTA
  constexpr int NS = 4 / TPQ;              // 16-dim slices (and MOVT planes) per thread
  constexpr int DIMS = 16 * NS;
  extern __shared__ __align__(128) unsigned char smem[];
  const int J = p.J;
  const DsqgSmem L(J, p.j_large, QB);
  unsigned char* s_q = smem + L.o_q;
  unsigned char* s_e = smem + L.o_e;
  float* s_qe = reinterpret_cast<float*>(smem + L.o_qe);
  float* s_sc = reinterpret_cast<float*>(smem + L.o_sc);
  float* s_pb = reinterpret_cast<float*>(smem + L.o_pb);
  int* s_off = reinterpret_cast<int*>(smem + L.o_off);
  float* s_pbase = reinterpret_cast<float*>(smem + L.o_pbase);
  float* s_pgain = reinterpret_cast<float*>(smem + L.o_pgain);
  __shared__ int s_count[2];

  const int64_t b = blockIdx.z;
  const int64_t h = blockIdx.y;
  const int64_t hk = h / p.kv_group;
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int sub = tid % TPQ;
  const int qi = tid / TPQ;
  // Queries [row_begin, N) (absolute positions); q, y, gate, out and lse rows
  // are addressed relative to row_begin.
  const int64_t n0 = p.row_begin + (int64_t)blockIdx.x * QB;
  const int64_t n = n0 + qi;
  const int64_t rb = p.row_begin;
  const int64_t n_last = (n0 + QB < p.N ? n0 + QB : p.N) - 1;

  // ---- stage Q tile, bf16(E), tables
  const uint32_t q_base = smem_u32(s_q), e_base = smem_u32(s_e);
  for (int i = tid; i < QB * 8; i += kThreads) {
    const int r = i >> 3, c = i & 7;
    const int64_t row = n0 + r < p.N ? n0 + r : p.N - 1;
    const uint4 v = *reinterpret_cast<const uint4*>(p.q + b * p.sqb + h * p.sqh + (row - rb) * p.sqn + c * 8);
    *reinterpret_cast<uint4*>(s_q + (tile_addr(q_base, r, c) - q_base)) = v;
  }
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
    *reinterpret_cast<uint4*>(s_e + (tile_addr(e_base, r, c) - e_base)) =
        make_uint4(packed[0], packed[1], packed[2], packed[3]);
  }
  for (int j = tid; j < J; j += kThreads) {
    s_pb[j] = p.pos_bias[j * p.spj + h * p.sph];
    s_off[j] = p.offsets[j];
  }
  for (int i = tid; i < p.j_large * 4; i += kThreads) {
    const int j = i >> 2, r = i & 3;
    s_pbase[i] = p.pbase[j * p.sbj + h * p.sbh + r];
    s_pgain[i] = p.pgain[j * p.sgj + h * p.sgh + r];
  }
  __syncthreads();
  if (tid == 0) {
    // Offsets ascend inside each band: the usable ones are a prefix of each band.
    int cs = 0, cl = 0;
    for (int j = 0; j < p.j_small; ++j) cs += (s_off[j] <= n_last);
    for (int j = p.j_small; j < J; ++j) cl += (s_off[j] <= n_last);
    s_count[0] = cs;
    s_count[1] = cl;
  }
  // ---- QE[QB][jp] = Q . bf16(E)^T on tensor cores (m16n8k16 tiles spread over the 8 warps)
  {
    constexpr int MT = QB / 16;
    const int g = lane >> 2, t4 = lane & 3;
    for (int mt = warp % MT; mt < MT; mt += 8) {
      uint32_t a[4][4];
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const int mi = lane >> 3, r = lane & 7;
        ldsm_x4(tile_addr(q_base, mt * 16 + (mi & 1) * 8 + r, ks * 2 + (mi >> 1)), a[ks][0], a[ks][1], a[ks][2],
                a[ks][3]);
      }
      const int nstep = 8 / MT > 0 ? 8 / MT : 1;  // warps sharing this m-tile
      for (int nt = MT >= 8 ? 0 : warp / MT; nt < L.jp / 8; nt += nstep) {
        float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          uint32_t b0, b1;
          ldsm_x2(tile_addr(e_base, nt * 8 + (lane & 7), ks * 2 + ((lane >> 3) & 1)), b0, b1);
          mma_bf16(c, a[ks], b0, b1);
        }
        float* row0 = s_qe + (mt * 16 + g) * L.qe_ld + nt * 8 + 2 * t4;
        float* row1 = row0 + 8 * L.qe_ld;
        row0[0] = c[0]; row0[1] = c[1];
        row1[0] = c[2]; row1[1] = c[3];
      }
    }
  }
  __syncthreads();
  const int count_small = s_count[0];
  const int count_large = s_count[1];

  const bool row_ok = n < p.N && n >= p.query_start;
  const int nq = (int)(n < p.N ? n : p.N - 1);
  const int d0 = sub * DIMS;
  float qs[DIMS];  // q, pre-scaled by 2^-K_i for the q6 field placement (exact)
  float qsum = 0.0f;
#pragma unroll
  for (int sl = 0; sl < NS; ++sl) {
    RowSlice<false> qr;
    qr.load(p.q + b * p.sqb + h * p.sqh + ((int64_t)nq - rb) * p.sqn + d0 + 16 * sl, true);
    float t[16];
    qr.to_f32(t);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      qsum += t[i];
      qs[16 * sl + i] = Q6 ? t[i] * __int_as_float((127 - q6_field_shift(i)) << 23) : t[i];
    }
  }

  // Per-thread bases; row offsets below are 32-bit (the host checks N * stride < 2^31).
  const uint8_t* kcb = p.kc + b * p.ccb + hk * p.cch + sub * (12 * NS);
  const uint8_t* vcb = p.vc + b * p.ccb + hk * p.cch + sub * (12 * NS);
  const uint16_t* ksb = p.ks + b * p.csb + hk * p.csh;
  const uint16_t* vsb = p.vs + b * p.csb + hk * p.csh;
  const __nv_bfloat16* kb = p.k + b * p.skb + hk * p.skh + d0;
  const __nv_bfloat16* vb = p.v + b * p.svb + hk * p.svh + d0;
  const float* zb = p.z + b * p.szb + hk * p.szh + sub * NS;
  const int cct = (int)p.cct, cst = (int)p.cst, skn = (int)p.skn, svn = (int)p.svn, szn = (int)p.szn;
  float* my_sc = s_sc + qi * L.sc_ld;
  const float* my_qe = s_qe + qi * L.qe_ld;
  const int nrow = row_ok ? nq : -1;  // src = nrow - off < 0 marks an invalid pair

  // ---- pass 1: scores of the live offsets (small band, then large band) and their max
  float m = -INFINITY;
  auto score_band = [&](int j_begin, int count, int slot0) {
    RowSlice<Q6> kn[NS];
    auto fetch = [&](int j, RowSlice<Q6> (&kr)[NS]) {
      const int src = nrow - s_off[j];
      const bool ok = src >= 0;
      const int r = ok ? src : 0;
#pragma unroll
      for (int sl = 0; sl < NS; ++sl) {
        if constexpr (Q6) kr[sl].load(kcb + r * cct + 12 * sl, ksb + r * cst, ok);
        else kr[sl].load(kb + r * skn + 16 * sl, ok);
      }
    };
    if (count > 0) fetch(j_begin, kn);
    for (int t = 0; t < count; ++t) {
      const int j = j_begin + t;
      RowSlice<Q6> kc[NS];
#pragma unroll
      for (int sl = 0; sl < NS; ++sl) kc[sl] = kn[sl];
      if (t + 1 < count) fetch(j + 1, kn);
      float p0 = 0.0f, p1 = 0.0f, stepk = 1.0f;
#pragma unroll
      for (int sl = 0; sl < NS; ++sl) {
        float kv[16];
        if constexpr (Q6) {
          uint32_t w3[3];
          kc[sl].to_scaled(kv, w3, stepk);
        } else {
          kc[sl].to_f32(kv);
        }
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          p0 = fmaf(qs[16 * sl + i], kv[i], p0);
          p1 = fmaf(qs[16 * sl + i + 1], kv[i + 1], p1);
        }
      }
      float part = Q6 ? ((p0 + p1) - 32.0f * qsum) * stepk : p0 + p1;
#pragma unroll
      for (int o = 1; o < TPQ; o <<= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      const float score = nrow - s_off[j] >= 0 ? (part + my_qe[j]) * 0.125f + s_pb[j] : -INFINITY;
      if (sub == 0) my_sc[slot0 + t] = score;
      m = fmaxf(m, score);
    }
  };
  score_band(0, count_small, 0);
  score_band(p.j_small, count_large, count_small);
  __syncwarp();

  // ---- pass 2: weights against the final max, V accumulation
  float acc[DIMS];
#pragma unroll
  for (int i = 0; i < DIMS; ++i) acc[i] = 0.0f;
  float l = 0.0f, wbias = 0.0f;  // wbias: sum of w * step_v (q6 offset correction)
  float corr_a[NS], corr_b[NS], yq[NS];
#pragma unroll
  for (int sl = 0; sl < NS; ++sl) {
    corr_a[sl] = corr_b[sl] = 0.0f;
    yq[sl] = p.y[b * p.syb + h * p.syh + ((int64_t)nq - rb) * p.syn + sub * NS + sl];
  }
  const float msafe = m == -INFINITY ? 0.0f : m;
  const int rot_a = p.plane_shift;
  auto value_band = [&](int j_begin, int count, int slot0, auto large_tag) {
    constexpr bool kLarge = decltype(large_tag)::value;
    RowSlice<Q6> vn[NS];
    float zn[NS];
    auto fetch = [&](int j, RowSlice<Q6> (&vr)[NS], float (&zr)[NS]) {
      const int src = nrow - s_off[j];
      const bool ok = src >= 0;
      const int r = ok ? src : 0;
#pragma unroll
      for (int sl = 0; sl < NS; ++sl) {
        if constexpr (Q6) vr[sl].load(vcb + r * cct + 12 * sl, vsb + r * cst, ok);
        else vr[sl].load(vb + r * svn + 16 * sl, ok);
        if constexpr (kLarge) zr[sl] = ok ? __ldg(zb + r * szn + sl) : 0.0f;
      }
    };
    if (count > 0) fetch(j_begin, vn, zn);
    for (int t = 0; t < count; ++t) {
      const int j = j_begin + t;
      RowSlice<Q6> vc[NS];
      float zc[NS];
#pragma unroll
      for (int sl = 0; sl < NS; ++sl) { vc[sl] = vn[sl]; zc[sl] = zn[sl]; }
      if (t + 1 < count) fetch(j + 1, vn, zn);
      const float score = my_sc[slot0 + t];
      if (score == -INFINITY) continue;  // uniform across the query's threads
      const float w = exp2f((score - msafe) * kLog2e);
      l += w;
#pragma unroll
      for (int sl = 0; sl < NS; ++sl) {
        float vv[16];
        float va = 0.0f, vb2 = 0.0f;  // value-domain channels of this slice's MOVT plane
        if constexpr (Q6) {
          float stepv;
          uint32_t w3[3];
          vc[sl].to_scaled(vv, w3, stepv);
          const float wv = w * stepv;
          if (sl == 0) wbias += wv;
#pragma unroll
          for (int i = 0; i < 16; ++i) acc[16 * sl + i] = fmaf(wv, vv[i], acc[16 * sl + i]);
          if constexpr (kLarge) {
            va = (q6_u_at(w3, rot_a) - 32.0f) * stepv;
            vb2 = (q6_u_at(w3, rot_a + 1) - 32.0f) * stepv;
          }
        } else {
          vc[sl].to_f32(vv);
#pragma unroll
          for (int i = 0; i < 16; ++i) acc[16 * sl + i] = fmaf(w, vv[i], acc[16 * sl + i]);
          if constexpr (kLarge) {
#pragma unroll
            for (int i = 0; i < 15; ++i) {
              if (i == rot_a) { va = vv[i]; vb2 = vv[i + 1]; }
            }
          }
        }
        if constexpr (kLarge) {
          // MOVT: rotate this slice's plane; accumulate rotated-minus-unrotated.
          const int jl = j - p.j_small;
          const int plane = sub * NS + sl;
          const float theta = s_pbase[jl * 4 + plane] + s_pgain[jl * 4 + plane] * yq[sl] * zc[sl];
          float sn, cs;
          __sincosf(theta, &sn, &cs);
          corr_a[sl] += w * ((cs - 1.0f) * va - sn * vb2);
          corr_b[sl] += w * (sn * va + (cs - 1.0f) * vb2);
        }
      }
    }
  };
  value_band(0, count_small, 0, std::false_type{});
  value_band(p.j_small, count_large, count_small, std::true_type{});

  // Fold the plane corrections in, undo the q6 field scaling and bias.
  // (All slices of a row share one scale, so wbias is per row.)
#pragma unroll
  for (int sl = 0; sl < NS; ++sl) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float v = Q6 ? acc[16 * sl + i] * __int_as_float((127 - q6_field_shift(i)) << 23) - 32.0f * wbias
                   : acc[16 * sl + i];
      if (i == rot_a) v += corr_a[sl];
      if (i == rot_a + 1) v += corr_b[sl];
      acc[16 * sl + i] = v;
    }
  }

  if (n >= p.N) return;
  float gain = 1.0f;
  if (p.gain != nullptr)
    gain = p.gain_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.gain)[h])
                       : reinterpret_cast<const float*>(p.gain)[h];
#pragma unroll
  for (int sl = 0; sl < NS; ++sl) {
    float o[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i] = l > 0.0f ? round_bf16(acc[16 * sl + i] / l) : 0.0f;
    if (p.gain != nullptr) {
#pragma unroll
      for (int i = 0; i < 16; ++i) o[i] = p.gain_bf16 ? round_bf16(o[i] * gain) : o[i] * gain;
    }
    if (p.gate != nullptr) {
      RowSlice<false> gs;
      gs.load(p.gate + b * p.sgtb + (n - rb) * p.sgtn + h * 64 + d0 + 16 * sl, true);
      float gv[16];
      gs.to_f32(gv);
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
    uint4* dst = reinterpret_cast<uint4*>(p.out + b * p.sob + h * p.soh + (n - rb) * p.son + d0 + 16 * sl);
    dst[0] = packed[0];
    dst[1] = packed[1];
  }
  if (p.lse != nullptr && sub == 0) {
    p.lse[b * p.slb + h * p.slh + (n - rb) * p.sln] = l > 0.0f ? m + logf(l) : -INFINITY;
  }
}

// Decode rows (a few query rows over a long q6 cache): one warp per (query
// row, head), lane j owning offset j (J <= 32), so the J K/V row gathers of a
// query are issued at once instead of one after another. Scores, a warp
// softmax, then every lane's weighted (MOVT-rotated) V row goes through
// shared memory and lane d sums dims d and d + 32. Same math as
// dsqg_fwd_kernel up to fp32 summation order.
constexpr int kDecodeWarps = 4;
__global__ void __launch_bounds__(32 * kDecodeWarps) dsqg_decode_kernel(const DsqgParams p) {
  __shared__ float s_v[kDecodeWarps][32][65];
  __shared__ float s_q[kDecodeWarps][64];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t h = (int64_t)blockIdx.x * kDecodeWarps + warp;
  if (h >= p.H) return;  // warp-uniform; the kernel has no block-wide barrier
  const int64_t rb = p.pos != nullptr ? *p.pos : p.row_begin, n = rb + blockIdx.y, b = blockIdx.z;
  const int64_t hk = h / p.kv_group;
  const __nv_bfloat16* qrow = p.q + b * p.sqb + h * p.sqh + (n - rb) * p.sqn;
  s_q[warp][lane] = __bfloat162float(qrow[lane]);
  s_q[warp][lane + 32] = __bfloat162float(qrow[lane + 32]);
  __syncwarp();
  const float* q = s_q[warp];

  const int j = lane;
  const bool live = j < p.J;
  const int64_t src = n - (live ? p.offsets[j] : 0);
  const bool ok = live && src >= 0 && n >= p.query_start;
  const int64_t srow = ok ? src : 0;
  float score = -INFINITY;
  if (ok) {
    const uint32_t* kw = reinterpret_cast<const uint32_t*>(p.kc + b * p.ccb + hk * p.cch + srow * p.cct);
    uint32_t w[13];
#pragma unroll
    for (int i = 0; i < 12; ++i) w[i] = __ldg(kw + i);
    w[12] = 0u;
    const float stepk = __half2float(__ushort_as_half(__ldg(p.ks + b * p.csb + hk * p.csh + srow * p.cst))) *
                        (1.0f / 31.0f);
    float d0 = 0.0f, d1 = 0.0f, e0 = 0.0f, e1 = 0.0f;
    const float* se = p.se + (int64_t)j * p.sej;
#pragma unroll
    for (int d = 0; d < 64; ++d) {
      const int bit = 6 * (d & 15), wd = 3 * (d >> 4) + (bit >> 5);
      const uint32_t f = __funnelshift_r(w[wd], w[wd + 1], bit & 31) & 63u;
      const float c = (float)((int)(f << 26) >> 26);
      const float e = round_bf16(__ldg(se + d * p.sed));
      if (d & 1) { d1 = fmaf(q[d], c, d1); e1 = fmaf(q[d], e, e1); }
      else { d0 = fmaf(q[d], c, d0); e0 = fmaf(q[d], e, e0); }
    }
    score = ((d0 + d1) * stepk + (e0 + e1)) * 0.125f + __ldg(p.pos_bias + (int64_t)j * p.spj + h * p.sph);
  }
  float m = score;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float wgt = ok ? exp2f((score - m) * kLog2e) : 0.0f;
  float l = wgt;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);

  float* my_v = s_v[warp][lane];
  if (ok) {
    const uint32_t* vw = reinterpret_cast<const uint32_t*>(p.vc + b * p.ccb + hk * p.cch + srow * p.cct);
    uint32_t w[13];
#pragma unroll
    for (int i = 0; i < 12; ++i) w[i] = __ldg(vw + i);
    w[12] = 0u;
    const float stepv = __half2float(__ushort_as_half(__ldg(p.vs + b * p.csb + hk * p.csh + srow * p.cst))) *
                        (1.0f / 31.0f);
    float vv[64];
#pragma unroll
    for (int d = 0; d < 64; ++d) {
      const int bit = 6 * (d & 15), wd = 3 * (d >> 4) + (bit >> 5);
      const uint32_t f = __funnelshift_r(w[wd], w[wd + 1], bit & 31) & 63u;
      vv[d] = (float)((int)(f << 26) >> 26) * stepv;
    }
#pragma unroll
    for (int d = 0; d < 64; ++d) my_v[d] = wgt * vv[d];
    if (j >= p.j_small) {
      // MOVT: rotate plane r (channels 16r + shift, 16r + shift + 1) of the
      // weighted row in place (the rotation is linear).
      const int jl = j - p.j_small;
      // y_pre rows are absolute positions when row_begin comes from the device.
      const float* yrow = p.y + b * p.syb + h * p.syh + (p.pos != nullptr ? n : n - rb) * p.syn;
      const float* zrow = p.z + b * p.szb + hk * p.szh + srow * p.szn;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const float theta = p.pbase[jl * p.sbj + h * p.sbh + r] + p.pgain[jl * p.sgj + h * p.sgh + r] * yrow[r] * zrow[r];
        float sn, cs;
        __sincosf(theta, &sn, &cs);
        float* pa = my_v + 16 * r + p.plane_shift;
        const float va = pa[0], vb = pa[1];
        pa[0] = cs * va - sn * vb;
        pa[1] = sn * va + cs * vb;
      }
    }
  } else {
#pragma unroll
    for (int d = 0; d < 64; ++d) my_v[d] = 0.0f;
  }
  __syncwarp();
  float acc[2] = {0.0f, 0.0f};
  const int rows = p.J < 32 ? p.J : 32;
  for (int r = 0; r < rows; ++r) {
    acc[0] += s_v[warp][r][lane];
    acc[1] += s_v[warp][r][lane + 32];
  }
  float gain = 1.0f;
  if (p.gain != nullptr)
    gain = p.gain_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.gain)[h])
                       : reinterpret_cast<const float*>(p.gain)[h];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int d = lane + 32 * k;
    float o = l > 0.0f ? round_bf16(acc[k] / l) : 0.0f;
    if (p.gain != nullptr) o = p.gain_bf16 ? round_bf16(o * gain) : o * gain;
    if (p.gate != nullptr) {
      const float gv = __bfloat162float(p.gate[b * p.sgtb + (n - rb) * p.sgtn + h * 64 + d]);
      const float sg = round_bf16(1.0f / (1.0f + expf(-gv)));
      o = p.gain_bf16 || p.gain == nullptr ? round_bf16(o * sg) : o * sg;
    }
    p.out[b * p.sob + h * p.soh + (n - rb) * p.son + d] = __float2bfloat16_rn(o);
  }
  if (p.lse != nullptr && lane == 0) p.lse[b * p.slb + h * p.slh + (n - rb) * p.sln] = l > 0.0f ? m + logf(l) : -INFINITY;
}

template <bool Q6, int TPQ>
int launch_dsqg(const DsqgParams& p, int64_t B, int64_t H, int64_t N, int J, int j_large, cudaStream_t stream) {
  constexpr int QB = kThreads / TPQ;
  const size_t smem = DsqgSmem(J, j_large, QB).bytes;
  dim3 grid((unsigned)((N - p.row_begin + QB - 1) / QB), (unsigned)H, (unsigned)B);
  if (grid.z > 65535 || grid.y > 65535) return DWARF_ERR_SHAPE;
  auto kernel = dsqg_fwd_kernel<Q6, TPQ>;
  if (smem > 48 * 1024 && cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem))
    return DWARF_ERR_LAUNCH;
  kernel<<<grid, kThreads, smem, stream>>>(p);
  return launch_status();
}

bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool a4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

}  // namespace
}  // namespace dwarf

using namespace dwarf;

extern "C" int dwarf_dsqg_fwd(const dwarf_dsqg_fwd_args* a, void* stream) {
  DWARF_CHECK_VERSION(a);
  if (a->kv_format != 0 && a->kv_format != 1) return DWARF_ERR_VALUE;
  if (a->head_dim != 64) return DWARF_ERR_SHAPE;
  if (a->B < 0 || a->H <= 0 || a->H_kv <= 0 || a->N < 0 || a->H % a->H_kv != 0) return DWARF_ERR_SHAPE;
  if (a->J < 1 || a->j_small < 0 || a->j_large < 0 || a->j_small + a->j_large != a->J || a->J > 512)
    return DWARF_ERR_SHAPE;
  if (a->plane_shift < 0 || a->plane_shift > 14) return DWARF_ERR_VALUE;
  if (a->row_begin < 0 || a->row_begin > a->N) return DWARF_ERR_SHAPE;
  if (a->B == 0 || a->N == 0 || a->row_begin == a->N) return DWARF_OK;
  if (!a->q || !a->out || !a->offsets || !a->pos_bias || !a->scale_embed || !a->y_pre || !a->z_pre)
    return DWARF_ERR_NULL;
  if (a->j_large > 0 && (!a->phase_base || !a->phase_gain)) return DWARF_ERR_NULL;
  const bool q6 = a->kv_format == 1;
  if (q6) {
    if (!a->k_codes || !a->v_codes || !a->k_scales || !a->v_scales) return DWARF_ERR_NULL;
    if (!a4(a->k_codes) || !a4(a->v_codes) || (a->ccb | a->cch | a->cct) % 4 != 0) return DWARF_ERR_ALIGN;
  } else {
    if (!a->k || !a->v) return DWARF_ERR_NULL;
    if (!a16(a->k) || !a16(a->v) || (a->skb | a->skh | a->skn | a->svb | a->svh | a->svn) % 8 != 0)
      return DWARF_ERR_ALIGN;
  }
  if (!a16(a->q) || !a16(a->out) || (a->sqb | a->sqh | a->sqn | a->sob | a->soh | a->son) % 8 != 0)
    return DWARF_ERR_ALIGN;
  if (a->gate != nullptr && (!a16(a->gate) || (a->sgb_ | a->sgn_) % 8 != 0)) return DWARF_ERR_ALIGN;
  if (a->head_gain != nullptr && a->head_gain_dtype != DWARF_F32 && a->head_gain_dtype != DWARF_BF16)
    return DWARF_ERR_DTYPE;

  // Row offsets inside the kernel are 32-bit.
  const int64_t lim = (int64_t)1 << 31;
  if (a->N * (q6 ? (a->cct > a->cst ? a->cct : a->cst) : (a->skn > a->svn ? a->skn : a->svn)) >= lim ||
      a->N * a->szn >= lim)
    return DWARF_ERR_SHAPE;
  DsqgParams p{};
  p.H = a->H; p.Hkv = a->H_kv; p.N = a->N;
  p.J = a->J; p.j_small = a->j_small; p.j_large = a->j_large;
  p.plane_shift = a->plane_shift;
  p.query_start = a->query_start < 0 ? 0 : a->query_start;
  p.kv_group = (int)(a->H / a->H_kv);
  p.q = (const __nv_bfloat16*)a->q; p.sqb = a->sqb; p.sqh = a->sqh; p.sqn = a->sqn;
  p.k = (const __nv_bfloat16*)a->k; p.skb = a->skb; p.skh = a->skh; p.skn = a->skn;
  p.v = (const __nv_bfloat16*)a->v; p.svb = a->svb; p.svh = a->svh; p.svn = a->svn;
  p.kc = a->k_codes; p.ks = a->k_scales; p.vc = a->v_codes; p.vs = a->v_scales;
  p.ccb = a->ccb; p.cch = a->cch; p.cct = a->cct; p.csb = a->csb; p.csh = a->csh; p.cst = a->cst;
  p.offsets = a->offsets;
  p.pos_bias = a->pos_bias; p.spj = a->spj; p.sph = a->sph;
  p.se = a->scale_embed; p.sej = a->sej; p.sed = a->sed;
  p.pbase = a->phase_base; p.sbj = a->sbj; p.sbh = a->sbh;
  p.pgain = a->phase_gain; p.sgj = a->sgj; p.sgh = a->sgh;
  p.y = a->y_pre; p.syb = a->syb; p.syh = a->syh; p.syn = a->syn;
  p.z = a->z_pre; p.szb = a->szb; p.szh = a->szh; p.szn = a->szn;
  p.out = (__nv_bfloat16*)a->out; p.sob = a->sob; p.soh = a->soh; p.son = a->son;
  p.lse = a->lse; p.slb = a->slb; p.slh = a->slh; p.sln = a->sln;
  p.gain = a->head_gain; p.gain_bf16 = a->head_gain_dtype == DWARF_BF16;
  p.gate = (const __nv_bfloat16*)a->gate; p.sgtb = a->sgb_; p.sgtn = a->sgn_;
  p.status = a->device_status;
  p.row_begin = a->row_begin;
  p.pos = a->pos;

  // 2 threads per query (32 dims each): half the per-pair bookkeeping of the
  // 4-thread layout. DWARF_DSQG_TPQ=4 selects the 4-thread layout.
  static const int tpq = [] {
    const char* e = getenv("DWARF_DSQG_TPQ");
    return (e && e[0] == '4') ? 4 : 2;
  }();
  cudaStream_t st = (cudaStream_t)stream;
  // q6 caches in the engine's own layout run on the resident-K/V kernel;
  // DWARF_DSQG_PATH=gather forces the gather kernel (read on every call).
  if (q6) {
    const char* path = getenv("DWARF_DSQG_PATH");
    if (!(path && path[0] == 'g') && p.row_begin == 0 && p.pos == nullptr) {
      const int rc = dsqg_resident_launch(p, a->B, st);
      if (rc != kNotApplicable) return rc;
    }
  }
  // A few query rows (decode steps) over a q6 cache: the one-warp-per-row
  // kernel (the only one that takes a device-side row_begin).
  const bool decode_shape = q6 && a->J <= 32 && a->N - p.row_begin <= 16;
  if (p.pos != nullptr && !decode_shape) return DWARF_ERR_VALUE;
  if (decode_shape) {
    const char* path = getenv("DWARF_DSQG_PATH");
    if (p.pos != nullptr || !(path && path[0] == 'g')) {
      dim3 grid((unsigned)((a->H + kDecodeWarps - 1) / kDecodeWarps), (unsigned)(a->N - p.row_begin), (unsigned)a->B);
      if (grid.z > 65535) return DWARF_ERR_SHAPE;
      dsqg_decode_kernel<<<grid, 32 * kDecodeWarps, 0, st>>>(p);
      return launch_status();
    }
  }
  if (q6) return tpq == 4 ? launch_dsqg<true, 4>(p, a->B, a->H, a->N, a->J, a->j_large, st)
                          : launch_dsqg<true, 2>(p, a->B, a->H, a->N, a->J, a->j_large, st);
  return tpq == 4 ? launch_dsqg<false, 4>(p, a->B, a->H, a->N, a->J, a->j_large, st)
                  : launch_dsqg<false, 2>(p, a->B, a->H, a->N, a->J, a->j_large, st);
}

