// bf16 GEMM on the 5th-generation tensor cores with fused epilogues.
//
// out = epilogue(A . B^T), A [M, K] and B [N, K] both K-major bf16 (x and a
// torch Linear weight), fp32 accumulation in tensor memory.
//
// Persistent, warp-specialised kernel, one CTA per SM:
//   warp 0      TMA producer: A tile [128 x 64] and B tile [BN x 64] per
//               k-block into an S-stage shared-memory ring (128-byte
//               swizzle, one mbarrier pair per stage);
//   warp 1      allocates tensor memory and issues tcgen05.mma
//               (M = 128, N = BN, K = 16 per instruction) from one thread;
//               tcgen05.commit frees a stage once its MMAs have read it and
//               marks an accumulator full after the tile's last k-block;
//   warps 2-5   epilogue: each thread owns one accumulator row (TMEM lane),
//               reads it with tcgen05.ld, applies the epilogue and stores.
// Two accumulator buffers (2 x BN columns of TMEM) let the epilogue of tile
// i overlap the MMAs of tile i + 1. Tiles are walked M-block-major so the
// CTAs working on one A block at a time share it through L2.
//
// Every mbarrier wait is bounded; a timeout sets a shared abort flag that
// ends every role's loop, records DWARF_DEVICE_TIMEOUT, waits (bounded) for
// the copies and MMAs already issued and releases tensor memory.
#include "common.cuh"
#include "q6_format.cuh"

#include "tma.cuh"

#include <type_traits>

namespace dwarf {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;  // bf16 elements per 128-byte swizzle row
constexpr int kGemmThreads = 320;  // TMA warp, MMA warp, 8 epilogue warps
constexpr uint32_t kWaitLimit = 1u << 24;

enum : int {
  kEpiStore = DWARF_GEMM_STORE,
  kEpiSwiglu = DWARF_GEMM_SWIGLU,
  kEpiRmsNorm = DWARF_GEMM_RESID_RMSNORM,
  kEpiQkvg = DWARF_GEMM_QKVG_PREP,
  kEpiLse = DWARF_GEMM_LSE
};

struct GemmEpi {
  const void* bias;
  int bias_bf16;
  __nv_bfloat16* out;
  int64_t ldo;
  int32_t* status;
  // residual + RMSNorm epilogue
  const __nv_bfloat16* resid;
  int64_t ldr;
  const void* norm_w;
  int norm_w_bf16;
  float eps;
  // qkvg + DSQG prep epilogue
  int T, heads;
  int64_t cache_len;  // rows per (b, h) in y / z / codes / scales
  const float* q_probe;
  const float* k_probe;
  float* y_pre;
  float* z_pre;
  uint8_t* k_codes;
  uint16_t* k_scales;
  uint8_t* v_codes;
  uint16_t* v_scales;
  // lm_head logsumexp / argmax epilogue
  float2* lse_part;
  float2* arg_part;
  const int64_t* targets;
  float* target_logit;
  const int64_t* pos;  // qkvg: optional device row offset of the cache
};

__device__ __forceinline__ uint32_t s32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile("{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}"
               : "=r"(done) : "r"(bar), "r"(parity) : "memory");
  return done != 0;
}
// Bounded wait; gives up (and raises the CTA's abort flag) after kWaitLimit
// polls or as soon as another role has aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  for (uint32_t it = 0; it < kWaitLimit; ++it) {
    if (mbar_try(bar, parity)) return true;
    if (*abort_flag) return false;
  }
  *abort_flag = 1;
  return false;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar) : "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, rows of
// 128 bytes in 8-row (1024-byte) atoms.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)(16 >> 4) << 16;    // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;  // stride byte offset: next 8-row atom
  d |= (uint64_t)1 << 46;            // descriptor version for sm_100
  d |= (uint64_t)2 << 61;            // 128-byte swizzle
  return d;
}
// Instruction descriptor, kind::f16: bf16 A and B (K-major), fp32 D.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---- CTA-pair (cluster of 2) helpers
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of the same variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// Arrive on a barrier of another CTA of the cluster (default .release.cta
// semantics: the signal orders this thread's prior tensor-memory reads, which
// tcgen05.wait::ld and the tcgen05 fence already completed; a cluster-scope
// release would also wait for the thread's outstanding global stores).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA load into this CTA's shared memory whose bytes complete on the
// leader's (rank 0) barrier at the same offset.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(map_rank(bar, 0)) : "memory");
}
__device__ __forceinline__ void tc_mma_pair(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n}"
      ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0u) : "memory");
}
// Arrives on the leader's own barrier once the pair's MMAs issued so far are done.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile("{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\ntcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
               ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(acc) : "memory");
}
// 16 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 64 consecutive fp32 columns of this thread's TMEM lane: two x32 loads and
// the wait in one asm statement, so no use of the registers can be scheduled
// before they are valid.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%64];\n"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%65];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr), "r"(taddr + 32) : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}
// Columns [c, c+16) and [c2, c2+16) (x16 each), one wait.
__device__ __forceinline__ void tmem_ld16x2(uint32_t t1, uint32_t t2, float (&a)[16], float (&b)[16]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%32];\n"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%33];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(t1), "r"(t2) : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) { a[i] = __uint_as_float(r[i]); b[i] = __uint_as_float(r[16 + i]); }
}
// 32 fp32 columns of this thread's TMEM lane (load + wait in one asm).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr) : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// 32 bf16 of a row (64 bytes) as four 16-byte loads (plain loads: the row may be rewritten in place).
__device__ __forceinline__ void load_row32(const __nv_bfloat16* p, uint4 (&w)[4]) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = q[i];
}
// 32 RMSNorm weights (fp32 or bf16) from column col.
__device__ __forceinline__ void load_w32(const void* w, int bf16, int col, float (&o)[32]) {
  if (bf16) {
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(w) + col);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 v = __ldg(p + j);
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        o[8 * j + 2 * k] = __uint_as_float(u[k] << 16);
        o[8 * j + 2 * k + 1] = __uint_as_float(u[k] & 0xffff0000u);
      }
    }
  } else {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(w) + col);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 v = __ldg(p + j);
      o[4 * j] = v.x; o[4 * j + 1] = v.y; o[4 * j + 2] = v.z; o[4 * j + 3] = v.w;
    }
  }
}
__device__ __forceinline__ void add_bias64(const void* bias, int bf16, int col, float (&v)[64]) {
  if (bf16) {
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(bias) + col);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint4 w = __ldg(p + j);
      const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        v[8 * j + 2 * k] += __uint_as_float(u[k] << 16);
        v[8 * j + 2 * k + 1] += __uint_as_float(u[k] & 0xffff0000u);
      }
    }
  } else {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(bias) + col);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float4 w = __ldg(p + j);
      v[4 * j] += w.x; v[4 * j + 1] += w.y; v[4 * j + 2] += w.z; v[4 * j + 3] += w.w;
    }
  }
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];"
               ::"l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(src) : "memory");
}

// (a0, a1) += (q0, q1) * (x, y) as one packed fp32x2 FMA (sm_100), each lane an IEEE fma.
__device__ __forceinline__ void fma2v(float& a0, float& a1, float q0, float q1, float x, float y) {
  asm("{\n.reg .b64 pa, pb, pc;\nmov.b64 pa, {%2, %3};\nmov.b64 pb, {%4, %5};\nmov.b64 pc, {%0, %1};\n"
      "fma.rn.f32x2 pc, pa, pb, pc;\nmov.b64 {%0, %1}, pc;\n}"
      : "+f"(a0), "+f"(a1)
      : "f"(q0), "f"(q1), "f"(x), "f"(y));
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const __nv_bfloat162 t = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&t);
}

// (a, b) rounded to bf16 and back with one packed conversion.
__device__ __forceinline__ void round_bf16_2(float& a, float& b) {
  const uint32_t w = pack2(a, b);
  a = __uint_as_float(w << 16);
  b = __uint_as_float(w & 0xffff0000u);
}
__device__ __forceinline__ void store16(__nv_bfloat16* dst, const float (&v)[16]) {
  uint4 w0 = make_uint4(pack2(v[0], v[1]), pack2(v[2], v[3]), pack2(v[4], v[5]), pack2(v[6], v[7]));
  uint4 w1 = make_uint4(pack2(v[8], v[9]), pack2(v[10], v[11]), pack2(v[12], v[13]), pack2(v[14], v[15]));
  reinterpret_cast<uint4*>(dst)[0] = w0;
  reinterpret_cast<uint4*>(dst)[1] = w1;
}

// Shared-memory stage of one CTA: A tile [128 x 64] + its part of the B tile
// (all BN rows alone, BN / 2 rows in a CTA pair).
template <int BN, int CTAS>
__host__ __device__ constexpr uint32_t gemm_stage_bytes() {
  return kBM * 128 + (BN / CTAS) * 128;
}
template <int EPI>
__host__ __device__ constexpr uint32_t gemm_table_bytes() {
  // RMSNorm partial sums (8 warps x 32 rows fp32) or the qkvg [2][4][64] probe tables.
  return EPI == DWARF_GEMM_RESID_RMSNORM ? 1024u : (EPI == DWARF_GEMM_QKVG_PREP ? 2048u : 0u);
}
template <int BN, int EPI, int CTAS>
__host__ __device__ constexpr int gemm_stages() {
  // As many stages as fit (at most 8) beside the staging boxes, barriers and tables.
  return (232448u - 1024u - 256u - gemm_table_bytes<EPI>() - (EPI != DWARF_GEMM_SWIGLU ? 8u * 4096u : 0u)) /
                     gemm_stage_bytes<BN, CTAS>() > 8u
             ? 8
             : (int)((232448u - 1024u - 256u - gemm_table_bytes<EPI>() -
                      (EPI != DWARF_GEMM_SWIGLU ? 8u * 4096u : 0u)) /
                     gemm_stage_bytes<BN, CTAS>());
}
template <int BN>
__host__ __device__ constexpr uint32_t gemm_tmem_cols() {
  return 2 * BN <= 256 ? 256u : 512u;
}
template <int EPI>
__host__ __device__ constexpr uint32_t gemm_staging_bytes() {
  return EPI != DWARF_GEMM_SWIGLU ? 8 * 4096 : 0;  // one 32 x 64 bf16 box per epilogue warp
}
template <int BN, int EPI, int CTAS>
__host__ __device__ constexpr size_t gemm_smem_bytes() {
  // 1 KB alignment slack, stages, staging boxes, barriers (256 B) and the
  // epilogue tables (RMSNorm partial sums or qkvg probes, at most 2 KB).
  return 1024 + (size_t)gemm_stages<BN, EPI, CTAS>() * gemm_stage_bytes<BN, CTAS>() + gemm_staging_bytes<EPI>() +
         256 + gemm_table_bytes<EPI>();
}

// CTAS = 2: a CTA pair (cluster of 2) computes 256 x BN tiles with
// tcgen05.mma.cta_group::2 issued by the even CTA (the leader). Each CTA
// loads its own 128 rows of A and BN / 2 rows of B; the operand halves stay in
// their own shared memory and the MMA reads both. The leader's full barriers
// count both CTAs' TMA bytes (the odd CTA's loads signal the leader's
// barrier), its commits arrive on the matching barriers of both CTAs, and the
// odd CTA's epilogue warps release the accumulator on the leader's barrier.
// No load is multicast: every CTA fetches only the bytes it keeps.
template <int BN, int EPI, int CTAS>
__global__ void __launch_bounds__(kGemmThreads, 1)
gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                 const __grid_constant__ CUtensorMap tmap_out, const __grid_constant__ CUtensorMap tmap_n,
                 const int M, const int N, const int K, const GemmEpi epi) {
  constexpr int S = gemm_stages<BN, EPI, CTAS>();
  constexpr uint32_t kStageA = kBM * 128, kStageB = (BN / CTAS) * 128;
  constexpr uint32_t kTmemCols = gemm_tmem_cols<BN>();
  constexpr uint32_t kIdesc = idesc_bf16(kBM * CTAS, BN);
  constexpr int kTileM = kBM * CTAS;  // rows per tile (both CTAs)
  extern __shared__ uint8_t gsm_raw[];
  const uint32_t raw = s32(gsm_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // 1024-byte aligned swizzle atoms
  uint8_t* gsm = gsm_raw + (base - raw);
  const uint32_t sA = base, sB = base + S * kStageA;
  const uint32_t sStage = base + S * (kStageA + kStageB);
  uint8_t* ctl = gsm + S * (kStageA + kStageB) + gemm_staging_bytes<EPI>();
  const uint32_t bar_full = s32(ctl), bar_empty = bar_full + 8 * S;
  const uint32_t bar_tfull = bar_empty + 8 * S, bar_tempty = bar_tfull + 16, bar_drain = bar_tempty + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ctl + 16 * S + 40);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(ctl + 16 * S + 44);
  constexpr uint32_t kAccStride = kTmemCols / 2;  // accumulator buffer a at column a * kAccStride

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = CTAS == 2 ? (int)cluster_rank() : 0;  // 0 = leader
  const int group = blockIdx.x / CTAS, groups = gridDim.x / CTAS;
  const int tiles_m = (M + kTileM - 1) / kTileM, tiles_n = N / BN;
  const int tiles = tiles_m * tiles_n;
  // i-th tile of this CTA (group). The RMSNorm epilogue needs whole rows, so
  // there a group owns M blocks and walks their tiles_n column tiles back to back.
  const int sub = EPI == kEpiRmsNorm ? tiles_n : 1;
  auto tile_at = [&](int i) { return (group + (i / sub) * groups) * sub + i % sub; };
  const int kblocks = (K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar_tfull + 8 * a, 1);
      mbar_init(bar_tempty + 8 * a, 8 * CTAS);  // one arrival per epilogue warp of the group
    }
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_a)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_b)) : "memory");
  }
  if (warp == 1) {
    if constexpr (CTAS == 2) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s32(tmem_slot)),
                   "r"(kTmemCols) : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s32(tmem_slot)),
                   "r"(kTmemCols) : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
  }
  tc_fence_before();
  if constexpr (CTAS == 2) cluster_sync();  // both CTAs' barriers exist before anyone signals them
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs of a pair)
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int i = 0; ok; ++i) {
        const int t = tile_at(i);
        if (t >= tiles) break;
        const int m0 = (t / tiles_n) * kTileM + kBM * rank, n0 = (t % tiles_n) * BN + (BN / CTAS) * rank;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const uint32_t s = it % S, ph = (it / S) & 1u;
          if (!(ok = mbar_wait(bar_empty + 8 * s, ph ^ 1u, abort_flag))) break;
          if constexpr (CTAS == 2) {
            // The MMA commit lands on the leader's empty barrier only; the
            // leader passes each release on to the odd CTA's barrier.
            if (rank == 0 && it >= (uint32_t)S) mbar_arrive_cluster(map_rank(bar_empty + 8 * s, 1));
            // The leader's full barrier expects both CTAs' bytes.
            if (rank == 0) mbar_expect_tx(bar_full + 8 * s, 2 * (kStageA + kStageB));
            tma_load_2d_pair(sA + s * kStageA, &tmap_a, kb * kBK, m0, bar_full + 8 * s);
            tma_load_2d_pair(sB + s * kStageB, &tmap_b, kb * kBK, n0, bar_full + 8 * s);
          } else {
            mbar_expect_tx(bar_full + 8 * s, kStageA + kStageB);
            tma_load_2d(sA + s * kStageA, &tmap_a, kb * kBK, m0, bar_full + 8 * s);
            tma_load_2d(sB + s * kStageB, &tmap_b, kb * kBK, n0, bar_full + 8 * s);
          }
        }
      }
      // Leave no copy in flight: the last S issued stages must have landed
      // (in a pair the leader's full barriers count the odd CTA's copies too).
      if (rank == 0)
        for (uint32_t j = it > (uint32_t)S ? it - S : 0; j < it; ++j) {
          const uint32_t s = j % S, ph = (j / S) & 1u;
          for (uint32_t w = 0; w < kWaitLimit && !mbar_try(bar_full + 8 * s, ph); ++w) {}
        }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer (the leader of a pair)
    if (lane == 0 && rank == 0) {
      uint32_t it = 0, tc = 0;
      bool ok = true;
      for (int i = 0; ok; ++i, ++tc) {
        const int t = tile_at(i);
        if (t >= tiles) break;
        const uint32_t a = tc & 1u, aph = (tc >> 1) & 1u;
        if (!(ok = mbar_wait(bar_tempty + 8 * a, aph ^ 1u, abort_flag))) break;
        tc_fence_after();
        const uint32_t d = tmem + a * kAccStride;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const uint32_t s = it % S, ph = (it / S) & 1u;
          if (!(ok = mbar_wait(bar_full + 8 * s, ph, abort_flag))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t da = smem_desc(sA + s * kStageA + kk * 32), db = smem_desc(sB + s * kStageB + kk * 32);
            if constexpr (CTAS == 2) tc_mma_pair(d, da, db, kIdesc, (kb | kk) != 0);
            else tc_mma(d, da, db, kIdesc, (kb | kk) != 0);
          }
          if constexpr (CTAS == 2) tc_commit_pair(bar_empty + 8 * s);
          else tc_commit(bar_empty + 8 * s);
        }
        if (ok) {
          if constexpr (CTAS == 2) tc_commit_pair(bar_tfull + 8 * a);
          else tc_commit(bar_tfull + 8 * a);
        }
      }
      // Drain: every MMA issued so far has completed once this commit lands.
      if constexpr (CTAS == 2) tc_commit_pair(bar_drain);
      else tc_commit(bar_drain);
      for (uint32_t w = 0; w < kWaitLimit && !mbar_try(bar_drain, 0); ++w) {}
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: warps 2..9. TMEM lane quarter = warp % 4;
    // the two warps of a quarter split the tile's columns.
    const int e = warp - 2, quarter = warp & 3, half = e >> 2;
    // Accumulator release: on the leader's barrier (remote for the odd CTA of a pair).
    auto release_acc = [&](uint32_t bar) {
      if (CTAS == 2 && rank != 0) mbar_arrive_cluster(map_rank(bar, 0));
      else mbar_arrive(bar);
    };
    if constexpr (EPI == kEpiQkvg) {
      // [q | k][probe pair][dim][2]: (p_{2r}[i], p_{2r+1}[i]) adjacent for packed FMAs
      float* sp = reinterpret_cast<float*>(ctl + 256);
      const int et = threadIdx.x - 64;  // 0..255 over the epilogue warps
      const int pr = et >> 6, dim = et & 63;  // probe, dim
      const int dst = ((pr >> 1) * 64 + dim) * 2 + (pr & 1);
      sp[dst] = epi.q_probe[et];
      sp[256 + dst] = epi.k_probe[et];
      asm volatile("bar.sync 5, 256;" ::: "memory");
    }
    uint32_t tc = 0;
    float ss = 0.0f;  // RMSNorm: running sum of squares of this thread's row slice
    // qkvg: device-side first cache row (a decode step replayed from a CUDA graph).
    const int64_t cache_row0 = (EPI == kEpiQkvg && epi.pos != nullptr) ? *epi.pos : 0;
    for (int i = 0;; ++i, ++tc) {
      const int t = tile_at(i);
      if (t >= tiles) break;
      const uint32_t a = tc & 1u, aph = (tc >> 1) & 1u;
      const int m0 = (t / tiles_n) * kTileM + kBM * rank, n0 = (t % tiles_n) * BN;
      // RMSNorm: the first residual chunk is loaded before waiting for the accumulator.
      uint4 rbuf[2][4];
      const int rrow = min(m0 + quarter * 32 + lane, M - 1);
      if constexpr (EPI == kEpiRmsNorm) load_row32(epi.resid + (int64_t)rrow * epi.ldr + n0 + half * (BN / 2), rbuf[0]);
      if (!mbar_wait(bar_tfull + 8 * a, aph, abort_flag)) break;
      // The accumulator-full commit lands on the leader; pass it on to the odd CTA.
      if (CTAS == 2 && rank == 0 && e == 0 && lane == 0) mbar_arrive_cluster(map_rank(bar_tfull + 8 * a, 1));
      tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(quarter * 32) << 16) + a * kAccStride;
      if constexpr (EPI == kEpiRmsNorm) {
        // Residual add + RMSNorm over whole rows (N <= 512, BN = 256): each
        // warp owns 32 rows x 128 columns of every column tile, in 32-column
        // chunks. Pass 1 writes v = x + addend (two chunks per 32 x 64 TMA
        // box) and accumulates the row's sum of squares, with the next
        // chunk's residual loaded while this one is processed; once the row
        // is complete, pass 2 reads v back (L2) from the rows this warp
        // itself stored, again one chunk ahead, and writes the normalised row.
        constexpr int CW = BN / 2;
        constexpr int NC = CW / 32;
        const uint32_t stg = sStage + e * 4096;
        uint8_t* stg_p = gsm + (stg - base);
        // Chunk k of a box: 16-byte pieces 4 (k & 1) + q of the 128-byte row.
        auto stage_chunk = [&](const CUtensorMap* map, const uint32_t (&pk)[16], int k, int col_box) {
          if ((k & 1) == 0) {
            if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
            __syncwarp();
          }
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4*>(stg_p + lane * 128 + (((4 * (k & 1) + q) ^ (lane & 7)) << 4)) =
                make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
          if (k & 1) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(map, stg, col_box, m0 + quarter * 32);
              asm volatile("cp.async.bulk.commit_group;" ::: "memory");
            }
          }
        };
        const int j = t % tiles_n;
        if (j == 0) ss = 0.0f;
        const __nv_bfloat16* rrow_p = epi.resid + (int64_t)rrow * epi.ldr + n0 + half * CW;
#pragma unroll
        for (int k = 0; k < NC; ++k) {
          if (k + 1 < NC) load_row32(rrow_p + 32 * (k + 1), rbuf[(k + 1) & 1]);
          float v[32];
          tmem_ld32(tbase + half * CW + 32 * k, v);
          if (k == NC - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) release_acc(bar_tempty + 8 * a);
          }
          uint32_t pk[16];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t u[4] = {rbuf[k & 1][q].x, rbuf[k & 1][q].y, rbuf[k & 1][q].z, rbuf[k & 1][q].w};
#pragma unroll
            for (int hh = 0; hh < 4; ++hh) {
              float a0 = v[8 * q + 2 * hh], a1 = v[8 * q + 2 * hh + 1];
              round_bf16_2(a0, a1);
              float lo = __uint_as_float(u[hh] << 16) + a0, hi = __uint_as_float(u[hh] & 0xffff0000u) + a1;
              round_bf16_2(lo, hi);
              ss = fmaf(lo, lo, ss);
              ss = fmaf(hi, hi, ss);
              pk[4 * q + hh] = pack2(lo, hi);
            }
          }
          stage_chunk(&tmap_out, pk, k, n0 + half * CW + 64 * (k >> 1));
        }
        if (j == tiles_n - 1) {
          float* ssb = reinterpret_cast<float*>(ctl + 256);
          ssb[e * 32 + lane] = ss;
          asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
          const float total = ssb[e * 32 + lane] + ssb[(e ^ 4) * 32 + lane];
          asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
          const float r = rsqrtf(total / (float)N + epi.eps);
          // This warp's v stores must have landed before it reads them back.
          if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;\nfence.proxy.async.global;" ::: "memory");
          __syncwarp();
          const __nv_bfloat16* vrow = epi.out + (int64_t)rrow * epi.ldo;
          const int nch = tiles_n * NC;  // this warp's chunks across the row
          auto col_of = [&](int kk) { return (kk / NC) * BN + half * CW + 32 * (kk % NC); };
          load_row32(vrow + col_of(0), rbuf[0]);
          auto step = [&](int kk, auto cur) {
            constexpr int C = decltype(cur)::value;
            if (kk + 1 < nch) load_row32(vrow + col_of(kk + 1), rbuf[C ^ 1]);
            const int col = col_of(kk);
            float wv[32];
            load_w32(epi.norm_w, epi.norm_w_bf16, col, wv);
            uint32_t pk[16];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint4 w4 = rbuf[C][q];
              const uint32_t u[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
              for (int hh = 0; hh < 4; ++hh)
                pk[4 * q + hh] = pack2((__uint_as_float(u[hh] << 16) * r) * wv[8 * q + 2 * hh],
                                       (__uint_as_float(u[hh] & 0xffff0000u) * r) * wv[8 * q + 2 * hh + 1]);
            }
            stage_chunk(&tmap_n, pk, kk % NC, (kk / NC) * BN + half * CW + 64 * ((kk % NC) >> 1));
          };
#pragma unroll 1
          for (int kk = 0; kk < nch; kk += 2) {  // nch is even
            step(kk, std::integral_constant<int, 0>{});
            step(kk + 1, std::integral_constant<int, 1>{});
          }
        }
      } else if constexpr (EPI == kEpiQkvg) {
        // One head (64 columns) per chunk; the tile lies inside one of the
        // q | k | v | gate sections. q and gate rows go out through the
        // staging box like epilogue 0; q and k rows give y / z (probe dots
        // over the bf16 row, scaled by rsqrt(|row|^2 + 64e-6)); k and v rows
        // are packed straight into the q6 cache.
        const int D = epi.heads * 64;
        const int sec = n0 / D;
        const float* s_probe = reinterpret_cast<const float*>(ctl + 256);  // [2][4][64]: q probes, k probes
        const int row = m0 + quarter * 32 + lane;
        const int b = row / epi.T, tt = row - b * epi.T;
        const uint32_t stg = sStage + e * 4096;
        uint8_t* stg_p = gsm + (stg - base);
#pragma unroll 1
        for (int k = 0; k < 2; ++k) {
          const int c = half * 128 + 64 * k;
          const int head = (n0 - sec * D + c) >> 6;
          float v[64];
          tmem_ld64(tbase + c, v);
          if (k == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) release_acc(bar_tempty + 8 * a);
          }
          add_bias64(epi.bias, epi.bias_bf16, n0 + c, v);
          // bf16 rounding once, as packed pairs: the words are the stored row and,
          // unpacked, the values every later step works on.
          uint32_t pw[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            pw[i] = pack2(v[2 * i], v[2 * i + 1]);
            v[2 * i] = __uint_as_float(pw[i] << 16);
            v[2 * i + 1] = __uint_as_float(pw[i] & 0xffff0000u);
          }
          const int64_t hrow = ((int64_t)b * epi.heads + head) * epi.cache_len + tt + cache_row0;
          if (sec == 0 || sec == 3) {
            if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint4 w = make_uint4(pw[4 * j], pw[4 * j + 1], pw[4 * j + 2], pw[4 * j + 3]);
              *reinterpret_cast<uint4*>(stg_p + lane * 128 + ((j ^ (lane & 7)) << 4)) = w;
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmap_out, stg, n0 + c, m0 + quarter * 32);
              asm volatile("cp.async.bulk.commit_group;" ::: "memory");
            }
          }
          if (sec <= 1 && row < M) {
            // probes stored as pairs (p0[i], p1[i]), (p2[i], p3[i]): one packed FMA per two probes
            const float4* pr = reinterpret_cast<const float4*>(s_probe + sec * 256);
            float ssq = 0.0f, d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int i2 = 0; i2 < 32; ++i2) {
              const float4 p01 = pr[i2];       // (p0[2 i2], p1[2 i2], p0[2 i2 + 1], p1[2 i2 + 1])
              const float4 p23 = pr[32 + i2];  // same for probes 2, 3
              fma2v(d[0], d[1], v[2 * i2], v[2 * i2], p01.x, p01.y);
              fma2v(d[0], d[1], v[2 * i2 + 1], v[2 * i2 + 1], p01.z, p01.w);
              fma2v(d[2], d[3], v[2 * i2], v[2 * i2], p23.x, p23.y);
              fma2v(d[2], d[3], v[2 * i2 + 1], v[2 * i2 + 1], p23.z, p23.w);
            }
#pragma unroll
            for (int i = 0; i < 64; ++i) ssq = fmaf(v[i], v[i], ssq);
            const float inv = rsqrtf(ssq + 1e-6f * 64.0f);
            float* dst = (sec == 0 ? epi.y_pre : epi.z_pre) + hrow * 4;
            *reinterpret_cast<float4*>(dst) = make_float4(d[0] * inv, d[1] * inv, d[2] * inv, d[3] * inv);
          }
          if ((sec == 1 || sec == 2) && row < M) {
            float amax = 0.0f;
#pragma unroll
            for (int i = 0; i < 64; ++i) amax = fmaxf(amax, fabsf(v[i]));
            const __half sh = q6_scale_from_amax(amax);
            const float qinv = q6_inv_step(__half2float(sh));
            // Rounding is monotonic, so when amax * inv (rounded) is below 31.5 every
            // product on the row rounds to |code| <= 31 and the clamp is the identity:
            // the common case (any fp16-normal scale) skips it. (The multiply and the
            // add stay separate scalar IEEE ops: a fused or packed pair rounds once and
            // can land on the other side of a .5 tie.)
            const bool clamp = !(__fmul_rn(amax, qinv) < 31.5f);
            uint32_t w[12];
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              uint32_t cc[16];
              // clamp(rint(x * inv), -31, 31) as q6_quantize (clamping first gives the same
              // code): adding 1.5 * 2^23 rounds to nearest-even into the low mantissa bits,
              // whose low six bits are the two's-complement code.
              if (!clamp) {
#pragma unroll
                for (int i = 0; i < 16; ++i)
                  cc[i] = __float_as_uint(__fadd_rn(__fmul_rn(v[16 * g + i], qinv), 12582912.0f)) & 63u;
              } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  const float qf = fminf(fmaxf(__fmul_rn(v[16 * g + i], qinv), -31.0f), 31.0f);
                  cc[i] = __float_as_uint(__fadd_rn(qf, 12582912.0f)) & 63u;
                }
              }
              w[3 * g] = cc[0] | cc[1] << 6 | cc[2] << 12 | cc[3] << 18 | cc[4] << 24 | cc[5] << 30;
              w[3 * g + 1] = cc[5] >> 2 | cc[6] << 4 | cc[7] << 10 | cc[8] << 16 | cc[9] << 22 | cc[10] << 28;
              w[3 * g + 2] = cc[10] >> 4 | cc[11] << 2 | cc[12] << 8 | cc[13] << 14 | cc[14] << 20 | cc[15] << 26;
            }
            uint4* cd = reinterpret_cast<uint4*>((sec == 1 ? epi.k_codes : epi.v_codes) + hrow * 48);
            cd[0] = make_uint4(w[0], w[1], w[2], w[3]);
            cd[1] = make_uint4(w[4], w[5], w[6], w[7]);
            cd[2] = make_uint4(w[8], w[9], w[10], w[11]);
            (sec == 1 ? epi.k_scales : epi.v_scales)[hrow] = __half_as_ushort(sh);
          }
        }
      } else if constexpr (EPI == kEpiLse) {
        // Online logsumexp and first-index argmax of this row's bf16-rounded
        // logits over the warp's half of the tile, 64 columns at a time, one
        // partial per (row, 128 columns): no exchange between the warps.
        constexpr int CW = BN / 2;
        constexpr float kLog2e = 1.4426950408889634f;
        const int row = m0 + quarter * 32 + lane;
        const int64_t tgt = (epi.targets != nullptr && row < M) ? epi.targets[row] : -1;
        float mx = -INFINITY, sm = 0.0f, best = -INFINITY;
        int bidx = 0;
#pragma unroll 1
        for (int c = half * CW; c < (half + 1) * CW; c += 64) {
          float v[64];
          tmem_ld64(tbase + c, v);
          if (c + 64 == (half + 1) * CW) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) release_acc(bar_tempty + 8 * a);
          }
          float cm = -INFINITY;
          int ci = 0;
#pragma unroll
          for (int j = 0; j < 64; j += 2) round_bf16_2(v[j], v[j + 1]);
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            if (v[j] > cm) { cm = v[j]; ci = j; }
          }
          if (cm > best) { best = cm; bidx = n0 + c + ci; }
          const float nm = fmaxf(mx, cm), nms = nm * kLog2e;
          float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll
          for (int j = 0; j < 64; j += 2) {
            acc0 += ex2_approx(fmaf(v[j], kLog2e, -nms));
            acc1 += ex2_approx(fmaf(v[j + 1], kLog2e, -nms));
          }
          sm = sm * ex2_approx((mx - nm) * kLog2e) + (acc0 + acc1);
          mx = nm;
          if (tgt >= n0 + c && tgt < n0 + c + 64) {
            const int k = (int)(tgt - n0 - c);
            float tv = 0.0f;
#pragma unroll
            for (int j = 0; j < 64; ++j) tv = j == k ? v[j] : tv;
            epi.target_logit[row] = tv;
          }
        }
        if (row < M) {
          const int64_t slot = ((int64_t)row * tiles_n + (t % tiles_n)) * 2 + half;
          epi.lse_part[slot] = make_float2(mx, sm);
          epi.arg_part[slot] = make_float2(best, __int_as_float(bidx));
        }
      } else if constexpr (EPI == kEpiStore) {
        // 64-column chunks: TMEM -> registers (+bias) -> bf16 rows in this
        // warp's 128-byte-swizzled staging box -> one TMA store of 32 x 64.
        constexpr int CW = BN / 2;
        const uint32_t stg = sStage + e * 4096;
        uint8_t* stg_p = gsm + (stg - base);
#pragma unroll 1
        for (int c = half * CW; c < (half + 1) * CW; c += 64) {
          float v[64];
          tmem_ld64(tbase + c, v);
          if (c + 64 == (half + 1) * CW) {  // last TMEM read of this tile by this warp
            tc_fence_before();
            __syncwarp();
            if (lane == 0) release_acc(bar_tempty + 8 * a);
          }
          if (epi.bias != nullptr) add_bias64(epi.bias, epi.bias_bf16, n0 + c, v);
          if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint4 w = make_uint4(pack2(v[8 * j], v[8 * j + 1]), pack2(v[8 * j + 2], v[8 * j + 3]),
                                       pack2(v[8 * j + 4], v[8 * j + 5]), pack2(v[8 * j + 6], v[8 * j + 7]));
            *reinterpret_cast<uint4*>(stg_p + lane * 128 + ((j ^ (lane & 7)) << 4)) = w;
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmap_out, stg, n0 + c, m0 + quarter * 32);
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          }
        }
      } else {
        // Tile columns [0, H) are up, [H, 2H) the matching gate columns;
        // 16-column chunks dealt alternately to the two warps of a quarter.
        constexpr int H = BN / 2;
        const int f0 = (t % tiles_n) * H;
        const int row = m0 + quarter * 32 + lane;
        constexpr int NCH = (H + 31) / 32;  // chunks per warp (the last may be absent for half 1)
#pragma unroll
        for (int k = 0; k < NCH; ++k) {
          const int c0 = half * 16 + 32 * k;
          const bool have = c0 < H;                      // warp-uniform
          const bool last = have && c0 + 32 >= H;        // this warp's last TMEM read of the tile
          float up[16], gt[16];
          if (have) tmem_ld16x2(tbase + c0, tbase + H + c0, up, gt);
          if (last) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) release_acc(bar_tempty + 8 * a);
          }
          if (!have) break;
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            // silu in fp32 with the hardware exp2 and a fast divide (the bf16
            // rounding after it absorbs the few-ulp fp32 difference).
            float u0 = up[i], u1 = up[i + 1], g0 = gt[i], g1 = gt[i + 1];
            round_bf16_2(u0, u1);
            round_bf16_2(g0, g1);
            float s0 = __fdividef(g0, 1.0f + __expf(-g0)), s1 = __fdividef(g1, 1.0f + __expf(-g1));
            round_bf16_2(s0, s1);
            up[i] = s0 * u0;
            up[i + 1] = s1 * u1;
          }
          if (row < M) store16(epi.out + (int64_t)row * epi.ldo + f0 + c0, up);
        }
      }
    }
    if (EPI != kEpiSwiglu && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
  }

  tc_fence_before();
  if constexpr (CTAS == 2) cluster_sync();  // no CTA leaves while its peer may still signal it
  else __syncthreads();
  if (*abort_flag && threadIdx.x == 0 && epi.status != nullptr) atomicExch(epi.status, DWARF_DEVICE_TIMEOUT);
  if (warp == 1) {
    tc_fence_after();
    if constexpr (CTAS == 2)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// ---------------------------------------------------------------- host side


// 2-D bf16 tensor map over rows x cols (row stride ld elements), box box_rows x
// box_cols (box_cols * 2 <= 128 bytes: one 128-byte swizzle row).
bool make_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t K, int64_t ld, int box_rows, int box_cols) {
  auto fn = tensormap_encoder();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int num_sms() {
  static int n = [] {
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v > 0 ? v : kNumSMs;
  }();
  return n;
}

template <int BN, int EPI, int CTAS>
int launch_gemm_impl(const dwarf_gemm_args* a, const GemmEpi& epi, cudaStream_t stream) {
  CUtensorMap ma, mb, mo;
  if (!make_map(&ma, a->a, a->M, a->K, a->lda, kBM, kBK) ||
      !make_map(&mb, a->b, a->N, a->K, a->ldb, BN / CTAS, kBK))
    return DWARF_ERR_LAUNCH;
  CUtensorMap mn = ma;
  // Output boxes of 32 rows x 64 columns (epilogues 0, 2 and 3).
  if (EPI != kEpiSwiglu && EPI != kEpiLse && !make_map(&mo, a->out, a->M, a->N, a->ldo, 32, 64))
    return DWARF_ERR_LAUNCH;
  if (EPI == kEpiSwiglu || EPI == kEpiLse) mo = ma;  // unused
  if (EPI == kEpiRmsNorm && !make_map(&mn, a->n_out, a->M, a->N, a->ldn, 32, 64)) return DWARF_ERR_LAUNCH;
  constexpr size_t smem = gemm_smem_bytes<BN, EPI, CTAS>();
  auto kernel = gemm_bf16_kernel<BN, EPI, CTAS>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return launch_status();
  // Work units (per CTA group): tiles, or whole M blocks for the RMSNorm epilogue.
  const int64_t tile_m = (int64_t)kBM * CTAS;
  const int64_t units = ((a->M + tile_m - 1) / tile_m) * (EPI == kEpiRmsNorm ? 1 : a->N / BN);
  const int64_t groups_max = num_sms() / CTAS;
  const int groups = (int)(units < groups_max ? units : groups_max);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(groups * CTAS));
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CTAS;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kernel, ma, mb, mo, mn, (int)a->M, (int)a->N, (int)a->K, epi) != cudaSuccess)
    return launch_status();
  return launch_status();
}

// CTA pairs (cta_group::2) unless DWARF_GEMM_CTAS=1 (read on every call).
template <int BN, int EPI>
int launch_gemm(const dwarf_gemm_args* a, const GemmEpi& epi, cudaStream_t stream) {
  const char* e = getenv("DWARF_GEMM_CTAS");
  if (e != nullptr && e[0] == '1') return launch_gemm_impl<BN, EPI, 1>(a, epi, stream);
  return launch_gemm_impl<BN, EPI, 2>(a, epi, stream);
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace dwarf

using namespace dwarf;

extern "C" int dwarf_gemm_bf16(const dwarf_gemm_args* a, void* stream) {
  DWARF_CHECK_VERSION(a);
  if (a->epilogue < DWARF_GEMM_STORE || a->epilogue > DWARF_GEMM_LSE) return DWARF_ERR_VALUE;
  if (a->M < 0 || a->N <= 0 || a->K <= 0 || a->K % 8 != 0) return DWARF_ERR_SHAPE;
  if (a->M > 0x7fffffffLL || a->N > 0x7fffffffLL || a->K > 0x7fffffffLL) return DWARF_ERR_SHAPE;
  if (a->M == 0) return DWARF_OK;
  const bool lse = a->epilogue == DWARF_GEMM_LSE;  // writes partials, not out
  if (!a->a || !a->b || (!lse && !a->out)) return DWARF_ERR_NULL;
  if (!al16(a->a) || !al16(a->b) || a->lda % 8 || a->ldb % 8 || a->lda < a->K || a->ldb < a->K ||
      (!lse && (!al16(a->out) || a->ldo % 8)))
    return DWARF_ERR_ALIGN;
  if (a->bias != nullptr && a->bias_dtype != DWARF_F32 && a->bias_dtype != DWARF_BF16) return DWARF_ERR_DTYPE;
  GemmEpi epi{a->bias, a->bias_dtype == DWARF_BF16, (__nv_bfloat16*)a->out, a->ldo, a->device_status,
              (const __nv_bfloat16*)a->resid, a->ldr, a->norm_w, a->norm_w_dtype == DWARF_BF16, a->eps,
              (int)a->T, a->heads, a->cache_len > 0 ? a->cache_len : a->T, a->q_probe, a->k_probe, a->y_pre,
              a->z_pre, a->k_codes, a->k_scales, a->v_codes, a->v_scales, (float2*)a->lse_part,
              (float2*)a->arg_part, a->targets, a->target_logit, a->pos};
  cudaStream_t st = (cudaStream_t)stream;
  if (lse) {
    if (a->N % 256 != 0) return DWARF_ERR_SHAPE;
    if (a->bias != nullptr) return DWARF_ERR_VALUE;
    if (!a->lse_part || !a->arg_part || (a->targets && !a->target_logit)) return DWARF_ERR_NULL;
    if ((reinterpret_cast<uintptr_t>(a->lse_part) | reinterpret_cast<uintptr_t>(a->arg_part)) & 7u)
      return DWARF_ERR_ALIGN;
    return launch_gemm<256, kEpiLse>(a, epi, st);
  }
  if (a->epilogue == DWARF_GEMM_QKVG_PREP) {
    if (a->heads <= 0 || a->N != 256LL * a->heads || (64LL * a->heads) % 256 != 0) return DWARF_ERR_SHAPE;
    if (a->T <= 0 || a->M % a->T != 0 || a->T > 0x7fffffffLL) return DWARF_ERR_SHAPE;
    if (!a->bias || !a->q_probe || !a->k_probe || !a->y_pre || !a->z_pre || !a->k_codes || !a->k_scales ||
        !a->v_codes || !a->v_scales)
      return DWARF_ERR_NULL;
    if (!al16(a->q_probe) || !al16(a->k_probe) || !al16(a->y_pre) || !al16(a->z_pre) || !al16(a->k_codes) ||
        !al16(a->v_codes) || !al16(a->bias) || a->ldo < a->N)
      return DWARF_ERR_ALIGN;
    return launch_gemm<256, kEpiQkvg>(a, epi, st);
  }
  if (a->epilogue == DWARF_GEMM_RESID_RMSNORM) {
    if (a->N != 256 && a->N != 512) return DWARF_ERR_SHAPE;
    if (!a->resid || !a->norm_w || !a->n_out) return DWARF_ERR_NULL;
    if (a->bias != nullptr) return DWARF_ERR_VALUE;
    if (!al16(a->resid) || !al16(a->n_out) || !al16(a->norm_w) || a->ldr % 8 || a->ldn % 8 || a->ldo < a->N ||
        a->ldr < a->N || a->ldn < a->N)
      return DWARF_ERR_ALIGN;
    if (a->norm_w_dtype != DWARF_F32 && a->norm_w_dtype != DWARF_BF16) return DWARF_ERR_DTYPE;
    return launch_gemm<256, kEpiRmsNorm>(a, epi, st);
  }
  if (a->epilogue == DWARF_GEMM_STORE) {
    if (a->ldo < a->N) return DWARF_ERR_SHAPE;
    if (a->N % 256 == 0) return launch_gemm<256, kEpiStore>(a, epi, st);
    if (a->N % 128 == 0) return launch_gemm<128, kEpiStore>(a, epi, st);
    return DWARF_ERR_SHAPE;
  }
  if (a->bias != nullptr) return DWARF_ERR_VALUE;
  const int h = a->swiglu_tile;
  if (a->N % (2 * h) != 0 || a->ldo < a->N / 2) return DWARF_ERR_SHAPE;
  if (h == 128) return launch_gemm<256, kEpiSwiglu>(a, epi, st);
  if (h == 80) return launch_gemm<160, kEpiSwiglu>(a, epi, st);
  if (h == 64) return launch_gemm<128, kEpiSwiglu>(a, epi, st);
  return DWARF_ERR_SHAPE;
}

namespace dwarf {
namespace {

// One warp per row: fold the row's (max, sum) and (max, first index) partials.
__global__ void __launch_bounds__(256) lse_reduce_kernel(const dwarf_lse_reduce_args a) {
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= a.M) return;
  constexpr float kLog2e = 1.4426950408889634f;
  const float2* lp = reinterpret_cast<const float2*>(a.lse_part) + row * a.parts;
  const float2* ap = reinterpret_cast<const float2*>(a.arg_part) + row * a.parts;
  float mx = -INFINITY, sm = 0.0f, best = -INFINITY;
  int bidx = 0x7fffffff;
  for (int64_t i = lane; i < a.parts; i += 32) {
    const float2 l = lp[i], g = ap[i];
    const float nm = fmaxf(mx, l.x);
    sm = sm * ex2_approx((mx - nm) * kLog2e) + l.y * ex2_approx((l.x - nm) * kLog2e);
    mx = nm;
    const int gi = __float_as_int(g.y);
    if (g.x > best || (g.x == best && gi < bidx)) { best = g.x; bidx = gi; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, mx, o), os = __shfl_xor_sync(0xffffffffu, sm, o);
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
    const float nm = fmaxf(mx, om);
    sm = (mx == -INFINITY ? 0.0f : sm * ex2_approx((mx - nm) * kLog2e)) +
         (om == -INFINITY ? 0.0f : os * ex2_approx((om - nm) * kLog2e));
    mx = nm;
    if (ob > best || (ob == best && oi < bidx)) { best = ob; bidx = oi; }
  }
  if (lane != 0) return;
  const float lse = mx + logf(sm);
  a.lse[row] = lse;
  if (a.argmax) a.argmax[row] = bidx;
  if (a.loss && a.targets) {
    const int64_t t = a.targets[row];
    a.loss[row] = t == a.ignore_index ? 0.0f : (t >= 0 && t < a.vocab ? lse - a.target_logit[row] : NAN);
  }
}

}  // namespace
}  // namespace dwarf

extern "C" int dwarf_lse_reduce(const dwarf_lse_reduce_args* a, void* stream) {
  DWARF_CHECK_VERSION(a);
  if (a->M < 0 || a->parts <= 0 || a->vocab <= 0) return DWARF_ERR_SHAPE;
  if (a->M == 0) return DWARF_OK;
  if (!a->lse_part || !a->arg_part || !a->lse) return DWARF_ERR_NULL;
  if (a->loss && (!a->targets || !a->target_logit)) return DWARF_ERR_NULL;
  const unsigned blocks = (unsigned)((a->M + 7) / 8);
  dwarf::lse_reduce_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(*a);
  return dwarf::launch_status();
}
