/*
 * dwarf_b200.h -- C ABI of the B200 (sm_100a) engine for the DWARF-v2
 * sparse-attention prefill path.
 *
 * Conventions shared by every entry point:
 *   - Arguments travel in a plain struct whose first field is `version`
 *     (DWARF_ABI_VERSION). Pointers are device pointers unless stated.
 *   - Strides are in ELEMENTS of the tensor they describe (as torch's
 *     Tensor.stride()), never bytes.
 *   - The entry point validates shapes, strides, dtypes and alignment on the
 *     host, launches on `stream`, and returns DWARF_OK (0) or a negative
 *     dwarf_status. It never synchronises, never throws and never allocates:
 *     the caller owns every output and every workspace buffer (the reference
 *     wrappers allocate outputs and scratch the same way, e.g.
 *     kernels/causal_ema_scan.py:282-287).
 *   - Kernels never report data errors: invalid (masked) rows produce exact
 *     zeros and LSE = -inf, as the reference kernels do
 *     (kernels/dsqg_attention_v22.py:845-851).
 *   - Kernels that spin on a flag written by another CTA bound the wait; when
 *     the bound is hit they record DWARF_DEVICE_TIMEOUT in the caller's
 *     `device_status` word (if given) instead of hanging.
 */
#ifndef DWARF_B200_H
#define DWARF_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DWARF_ABI_VERSION 1

typedef enum {
  DWARF_OK = 0,
  DWARF_ERR_VERSION = -1,      /* args->version != DWARF_ABI_VERSION          */
  DWARF_ERR_NULL = -2,         /* a required pointer is NULL                  */
  DWARF_ERR_SHAPE = -3,        /* inconsistent or unsupported sizes           */
  DWARF_ERR_STRIDE = -4,       /* unsupported layout                          */
  DWARF_ERR_ALIGN = -5,        /* pointer/stride misaligned for the kernel    */
  DWARF_ERR_DTYPE = -6,        /* unsupported dtype code                      */
  DWARF_ERR_WORKSPACE = -7,    /* workspace missing or too small              */
  DWARF_ERR_LAUNCH = -8,       /* cudaGetLastError() after the launch         */
  DWARF_ERR_VALUE = -9,        /* bad scalar argument                         */
  DWARF_ERR_SCRATCH_LIMIT = -10 /* problem needs more than the built-in scratch */
} dwarf_status;

/* Device-side status words written by kernels with bounded waits. */
#define DWARF_DEVICE_OK 0
#define DWARF_DEVICE_TIMEOUT 1

typedef enum {
  DWARF_F32 = 0,
  DWARF_BF16 = 1,
  DWARF_F16 = 2
} dwarf_dtype;

/* Human-readable name of a dwarf_status (static string). */
const char* dwarf_status_string(int status);
/* Returns DWARF_ABI_VERSION of the loaded library. */
int dwarf_abi_version(void);

/* ------------------------------------------------------------------------
 * Causal EMA scan.
 *
 * Replaces causal_ema_scan() -> _CausalEMAFn.forward -> _fwd_local/_fwd_carry/
 * _fwd_apply (kernels/causal_ema_scan.py:541-567, 265-313, 73-155):
 *     y[b,t,d] = alpha_d * x[b,t,d] + (1 - alpha_d) * y[b,t-1,d],  y[b,-1,d] = 0
 * with an fp32 state and y stored in the dtype of x. One launch, one read of
 * x and one write of y: a chunked scan whose chunks are chained by decoupled
 * look-back through `workspace`.
 *
 * alpha: fp32 device pointer, one scalar (alpha_per_channel = 0) or `width`
 * values. When clamp != 0 every alpha is clamped to [floor, ceiling] first,
 * exactly as the reference scalar API does (causal_ema_scan.py:274).
 * ---------------------------------------------------------------------- */
typedef struct {
  int32_t version;
  int32_t dtype;              /* dtype of x and y: DWARF_F32 or DWARF_BF16  */
  const void* x;              /* [batch, seq_len, width]                    */
  void* y;                    /* [batch, seq_len, width]                    */
  int64_t batch, seq_len, width;
  int64_t sxb, sxn, sxd;      /* element strides of x                       */
  int64_t syb, syn, syd;      /* element strides of y                       */
  const float* alpha;
  int32_t alpha_per_channel;
  int32_t clamp;
  float floor_, ceiling;
  void* workspace;            /* dwarf_ema_scan_workspace_bytes() bytes     */
  int64_t workspace_bytes;
  int32_t* device_status;     /* optional; set to DWARF_DEVICE_TIMEOUT      */
  const float* init_state;    /* optional fp32 [batch, width]: y[-1] (else 0) */
  float* final_state;         /* optional fp32 [batch, width]: the fp32 state
                                 after token seq_len-1 (may not alias init)  */
  uint32_t wait_limit;        /* polls before a look-back wait gives up and
                                 records DWARF_DEVICE_TIMEOUT (0: the default,
                                 about 0.3-1 s)                              */
  int32_t test_tag_skew;      /* testing only, 0 in normal use: nonzero makes
                                 readers expect a record tag that no writer
                                 produces, so every look-back wait runs out
                                 (exercises the bounded-wait path without a
                                 fault; the output is then not valid)        */
} dwarf_ema_scan_args;

int64_t dwarf_ema_scan_workspace_bytes(int64_t batch, int64_t seq_len, int64_t width,
                                       int32_t dtype);
int dwarf_ema_scan(const dwarf_ema_scan_args* args, void* stream);

/* Gradient of the causal EMA scan with respect to alpha.
 *
 * Replaces the COMPUTE_DA part of _bwd_apply (kernels/causal_ema_scan.py:204-260,
 * launched by _CausalEMAFn.backward :315-364):
 *     da[d] = sum_{b,t} s[b,t,d] * (x[b,t,d] - y[b,t-1,d]),   y[b,-1,d] = 0
 * where s is the reverse-time state s[t] = dy[t] + (1 - alpha_d) s[t+1].
 * The caller passes g = alpha_d * s, which is exactly the input gradient dx
 * (dwarf_ema_scan run over time-reversed dy), in fp32; the kernel divides each
 * channel's partial sum by alpha_d. x and y (the forward output) are in
 * `dtype`. alpha_per_channel = 0: one alpha and one output value (summed over
 * channels too); 1: `width` alphas and `width` outputs. `da` is overwritten
 * (zeroed on the stream, then accumulated with atomics, so the summation order
 * and the last bits vary between runs).
 * ---------------------------------------------------------------------- */
typedef struct {
  int32_t version;
  int32_t dtype;              /* dtype of x and y: DWARF_F32 or DWARF_BF16  */
  const void* x;              /* [batch, seq_len, width]                    */
  const void* y;              /* [batch, seq_len, width] forward output     */
  const float* g;             /* [batch, seq_len, width] fp32 alpha * state */
  int64_t batch, seq_len, width;
  int64_t sxb, sxn, sxd;      /* element strides of x                       */
  int64_t syb, syn, syd;      /* element strides of y                       */
  int64_t sgb, sgn, sgd;      /* element strides of g                       */
  const float* alpha;         /* fp32: 1 value or `width` values            */
  int32_t alpha_per_channel;
  int32_t pad_;
  float* da;                  /* fp32 [1] or [width]                        */
} dwarf_ema_grad_alpha_args;

int dwarf_ema_scan_grad_alpha(const dwarf_ema_grad_alpha_args* args, void* stream);

/* Causal EMA scan that allocates nothing and needs no caller workspace.
 *
 * No counterpart in the reference: this entry point exists for callers that
 * cannot allocate device memory at the point of the call -- for example code
 * running inside an allocator-less runtime, a plugin whose host forbids
 * cudaMalloc on its hot path, or an embedder that pre-sizes all device memory
 * up front. It computes exactly what dwarf_ema_scan computes (same kernel),
 * but keeps its look-back scratch in a fixed array that lives inside the
 * library (DWARF_EMA_NOALLOC_SCRATCH_BYTES per GPU that loads the library,
 * held until the process exits). The caller still passes x, y and alpha;
 * args->workspace and args->workspace_bytes are ignored.
 *
 *  - Size limit: problems whose scratch need (dwarf_ema_scan_workspace_bytes)
 *    exceeds DWARF_EMA_NOALLOC_SCRATCH_BYTES are rejected with
 *    DWARF_ERR_SCRATCH_LIMIT before anything is launched. 8 MiB covers e.g.
 *    B=16, T=2048, D=512 in fp32 or bf16.
 *  - Set-up: the first call on each device looks up the array's device
 *    address (cudaGetSymbolAddress) with that device current; make that
 *    first call before any stream capture begins.
 *  - Sharing: every call on a device uses the same array. Each call clears
 *    the part it uses (cudaMemsetAsync on its stream) before launching, so
 *    calls ordered on one stream are independent, but calls that can overlap
 *    on the GPU (different streams, or several host threads) race on the
 *    array and must be serialised by the caller.
 *  - Calls no cudaMalloc, cudaFree or other allocating routine. */
#define DWARF_EMA_NOALLOC_SCRATCH_BYTES (8 * 1024 * 1024)
int dwarf_ema_scan_noalloc(const dwarf_ema_scan_args* args, void* stream);


/* ------------------------------------------------------------------------
 * q6 KV codec (no reference counterpart: the reference declares a packed-KV
 * mode unimplemented, kernels/dsqg_attention_v22.py:467,473-476).
 *
 * One row = one (b, h, t) head vector of 64 values.
 *   amax  = max_d |x_d|                         (fp32)
 *   s     = fp16(min(amax, 65504))              (round to nearest even)
 *   inv   = 31 / float(s)                       (IEEE fp32 division)
 *   c_d   = clamp(rint(x_d * inv), -31, 31)     (fp32 multiply, RNE; s == 0 -> 0)
 *   bytes = 16 groups of 4 codes, each group 3 bytes little-endian:
 *           w = u0 | u1 << 6 | u2 << 12 | u3 << 18, u = c & 63 (6-bit two's
 *           complement); row = 48 bytes.
 *   dequant x^_d = float(c_d) * (float(s) / 31)
 * Codes [rows][48] u8, scales [rows] fp16, rows addressed (b, h, t) by strides.
 * ---------------------------------------------------------------------- */
typedef struct {
  int32_t version;
  int32_t dtype;              /* dtype of x: DWARF_BF16 or DWARF_F32        */
  const void* x;              /* [B, H, T, 64]                              */
  int64_t B, H, T;
  int64_t sxb, sxh, sxt;      /* element strides of x; dim stride must be 1 */
  uint8_t* codes;             /* [B, H, T, 48]                              */
  int64_t scb, sch, sct;      /* byte strides of codes rows (multiple of 16)*/
  uint16_t* scales;           /* fp16 bits [B, H, T]                        */
  int64_t ssb, ssh, sst;      /* element strides of scales                  */
} dwarf_q6_pack_args;

typedef struct {
  int32_t version;
  int32_t out_dtype;          /* DWARF_F32 or DWARF_BF16                    */
  const uint8_t* codes;
  int64_t B, H, T;
  int64_t scb, sch, sct;
  const uint16_t* scales;
  int64_t ssb, ssh, sst;
  void* x;                    /* [B, H, T, 64] output                       */
  int64_t sxb, sxh, sxt;
} dwarf_q6_unpack_args;

int dwarf_q6_pack(const dwarf_q6_pack_args* args, void* stream);
int dwarf_q6_unpack(const dwarf_q6_unpack_args* args, void* stream);

/* ------------------------------------------------------------------------
 * DSQG lattice attention forward.
 *
 * Replaces dsqg_attention_v18_grouped -> _DSQGV18GroupedFn.forward ->
 * _fwd_v22_online (kernels/dsqg_attention_v22.py:2691-2777, 2197-2352,
 * 698-860) for grouped_mode "baseline". For every query n and offset j
 * (canonical order: small offsets then large), src = n - off[j]:
 *   score = (q_n . (k_src + bf16(E_j))) / sqrt(64) + pos_bias[j, h]
 * online softmax over valid (src >= 0) offsets, accumulating v_src, where for
 * j >= j_small the four MOVT planes (a_r = 16 r + plane_shift, a_r + 1) of
 * v_src are rotated by theta = phase_base[j',h,r] + phase_gain[j',h,r] *
 * y_pre[n,r] * z_pre[src,r], j' = j - j_small. Rows with no valid offset
 * produce exact zeros and LSE = -inf.
 *
 * K/V come either as bf16 tensors (kv_format 0, the reference's layout,
 * any strides) or as a q6 cache (kv_format 1, dwarf_q6_pack layout).
 * head_dim must be 64; GQA (H % H_kv == 0) is supported.
 *
 * Optional fused epilogue (the module's `out * if_gain` and
 * `* sigmoid(content_gate)`, dsqg_attention_v22.py:3285-3289), with the
 * module's bf16 rounding points: o = bf16(acc/l); if head_gain:
 * o = bf16(o * head_gain[h]); if gate: o = bf16(o * bf16(sigmoid(gate))).
 * ---------------------------------------------------------------------- */
typedef struct {
  int32_t version;
  int32_t kv_format;              /* 0 = bf16 K/V, 1 = q6 cache           */
  int64_t B, H, H_kv, N;
  int32_t head_dim;               /* must be 64                           */
  int32_t J, j_small, j_large;
  int32_t plane_shift;
  int32_t query_start;            /* rows < query_start are written as 0  */
  const void* q;                  /* bf16 [B, H, N, 64]                   */
  int64_t sqb, sqh, sqn;          /* element strides; dim stride 1        */
  const void* k;                  /* bf16 [B, H_kv, N, 64] (kv_format 0)  */
  int64_t skb, skh, skn;
  const void* v;
  int64_t svb, svh, svn;
  const uint8_t* k_codes;         /* q6 (kv_format 1)                     */
  const uint16_t* k_scales;
  const uint8_t* v_codes;
  const uint16_t* v_scales;
  int64_t ccb, cch, cct;          /* byte strides of code rows (K and V)  */
  int64_t csb, csh, cst;          /* element strides of scales (K and V)  */
  const int32_t* offsets;         /* [J], device                          */
  const float* pos_bias;          /* [J, H]                               */
  int64_t spj, sph;
  const float* scale_embed;       /* [J, 64]                              */
  int64_t sej, sed;
  const float* phase_base;        /* [j_large, H, 4] (last dim stride 1)  */
  int64_t sbj, sbh;
  const float* phase_gain;        /* [j_large, H, 4]                      */
  int64_t sgj, sgh;
  const float* y_pre;             /* [B, H, N, 4] (last dim stride 1)     */
  int64_t syb, syh, syn;
  const float* z_pre;             /* [B, H_kv, N, 4]                      */
  int64_t szb, szh, szn;
  void* out;                      /* bf16 [B, H, N, 64] by strides        */
  int64_t sob, soh, son;
  float* lse;                     /* optional fp32 [B, H, N]              */
  int64_t slb, slh, sln;
  const void* head_gain;          /* optional [H], dtype head_gain_dtype  */
  int32_t head_gain_dtype;        /* DWARF_F32 or DWARF_BF16              */
  const void* gate;               /* optional bf16 [B, N, H*64] view      */
  int64_t sgb_, sgn_;             /* element strides (b, n); h*64+d is +1 */
  int32_t* device_status;         /* optional; set to DWARF_DEVICE_TIMEOUT */
  int64_t row_begin;              /* compute queries [row_begin, N) only; q,
                                     y_pre, gate, out and lse rows are then
                                     relative to row_begin (decode: N-1)  */
  const int64_t* pos;             /* optional device int64 P (decode step):
                                     row_begin = P at run time and N = P +
                                     (N - row_begin) of the call; y_pre
                                     rows are then absolute positions (it
                                     lives in the cache); q6 K/V, J <= 32,
                                     at most 16 rows                      */
} dwarf_dsqg_fwd_args;

int dwarf_dsqg_fwd(const dwarf_dsqg_fwd_args* args, void* stream);

/* ------------------------------------------------------------------------
 * DSQG lattice attention backward (bf16 K/V).
 *
 * Replaces _DSQGV18GroupedFn.backward (kernels/dsqg_attention_v22.py:2354-2552)
 * with its kernels _compute_D_v18_grouped, _bwd_dq_v18_grouped and
 * _bwd_dkdv_v18_grouped (:1263-2196): given dO and the forward's output and
 * natural-log lse, with p = exp(score - lse), dp = dO . v~ (v~ the MOVT-rotated
 * value), delta = dO . O and ds = p (dp - delta):
 *   dq[n]  = (1/8) sum_j ds (k[n-off_j] + bf16(E_j))
 *   dk[s]  = (1/8) sum_j ds q[s+off_j]          (over the query heads of s's KV head)
 *   dv[s]  = sum_j p R(theta)^T dO[s+off_j]
 *   dtheta = p (dO_b v~_a - dO_a v~_b) per plane (a, b); dy_pre[n,r] += dtheta *
 *   gain * z, dz_pre[s,r] += dtheta * gain * y, d phase_base += dtheta,
 *   d phase_gain += dtheta * y * z;
 * ds itself is written to `ds` [B, H, N, J] (0 for invalid pairs; pairs whose
 * offset reaches before token 0 for a whole warp of queries are not written,
 * so the caller zero-fills ds) for the caller's d pos_bias = sum_{b,n} ds and
 * d scale_embed = (1/8) sum_{b,h,n} ds q.
 * Layout: every tensor contiguous; head_dim 64; plane_shift <= 14; tables fp32
 * as in dwarf_dsqg_fwd_args (pos_bias [J,H], scale_embed [J,64], phase tables
 * [j_large,H,4]). Two launches: the query-side kernel (dq, dy_pre, ds, delta,
 * phase-table gradients; d_phase_* are zeroed on the stream first) then the
 * key-side kernel (dk, dv, dz_pre), each output written by one thread.
 * ---------------------------------------------------------------------- */
typedef struct {
  int32_t version;
  int32_t J, j_small, j_large, plane_shift, query_start;
  int64_t B, H, H_kv, N;
  const void* q;              /* bf16 [B, H, N, 64]                         */
  const void* k;              /* bf16 [B, H_kv, N, 64]                      */
  const void* v;              /* bf16 [B, H_kv, N, 64]                      */
  const void* out;            /* bf16 [B, H, N, 64] forward output          */
  const void* dout;           /* bf16 [B, H, N, 64]                         */
  const float* lse;           /* [B, H, N] natural-log lse of the forward   */
  const int32_t* offsets;     /* [J]                                        */
  const float* pos_bias;      /* [J, H]                                     */
  const float* scale_embed;   /* [J, 64]                                    */
  const float* phase_base;    /* [j_large, H, 4]                            */
  const float* phase_gain;    /* [j_large, H, 4]                            */
  const float* y_pre;         /* [B, H, N, 4]                               */
  const float* z_pre;         /* [B, H_kv, N, 4]                            */
  void* dq;                   /* bf16 [B, H, N, 64]                         */
  void* dk;                   /* bf16 [B, H_kv, N, 64]                      */
  void* dv;                   /* bf16 [B, H_kv, N, 64]                      */
  float* dy_pre;              /* [B, H, N, 4]                               */
  float* dz_pre;              /* [B, H_kv, N, 4]                            */
  float* ds;                  /* [B, H, N, J], zero-filled by the caller    */
  float* delta;               /* [B, H, N] written (dO . O)                 */
  float* d_phase_base;        /* [j_large, H, 4] overwritten                */
  float* d_phase_gain;        /* [j_large, H, 4] overwritten                */
} dwarf_dsqg_bwd_args;

int dwarf_dsqg_bwd(const dwarf_dsqg_bwd_args* args, void* stream);

/* ------------------------------------------------------------------------
 * DSQG QKV prep: the per-row work between the qkvg projection and the DSQG
 * kernel, fused into one pass over the projection output.
 *
 * Replaces the probe projections of DSQGAttentionV19.forward
 * (kernels/dsqg_attention_v22.py:3231-3254):
 *   y_pre[b,h,n,r] = (q . qp_r) / sqrt(|q|^2 + 1e-6*64)
 *   z_pre[b,h,n,r] = (k . kp_r) / sqrt(|k|^2 + 1e-6*64)
 * with qp/kp the L2-normalised probes [4][64] (fp32), and optionally packs K
 * and V rows into the q6 cache (dwarf_q6_pack format) in the same pass.
 * ---------------------------------------------------------------------- */
typedef struct {
  int32_t version;
  int32_t pack_q6;                /* 1: also write K/V q6 codes + scales  */
  int64_t B, H, H_kv, N;
  const void* q;                  /* bf16 [B, H, N, 64]                   */
  int64_t sqb, sqh, sqn;
  const void* k;                  /* bf16 [B, H_kv, N, 64]                */
  int64_t skb, skh, skn;
  const void* v;                  /* bf16 [B, H_kv, N, 64] (pack_q6 only) */
  int64_t svb, svh, svn;
  const float* q_probe;           /* [4][64]                              */
  const float* k_probe;           /* [4][64]                              */
  float* y_pre;                   /* [B, H, N, 4] contiguous              */
  float* z_pre;                   /* [B, H_kv, N, 4] contiguous           */
  uint8_t* k_codes;               /* [B, H_kv, N, 48] contiguous          */
  uint16_t* k_scales;             /* [B, H_kv, N] contiguous              */
  uint8_t* v_codes;
  uint16_t* v_scales;
} dwarf_dsqg_prep_args;

int dwarf_dsqg_prep(const dwarf_dsqg_prep_args* args, void* stream);

/* ------------------------------------------------------------------------
 * NPCI magnitude-aware rotation of head vectors (64 values per row).
 *
 * Replaces npci_rotate (kernels/dsqg_attention_v22.py:223-254) and
 * _magnitude_aware_rotate (kernels/hierarchical_sparse_attn_v18_hisa.py:99-125):
 *   x' = x (+ addend, rounded to the I/O dtype, when addend != NULL)
 *   u = x'/max(|x'|,1e-12); p = d - (d.u) u; active = |p| > |x'| 1e-7
 *   angle = theta[h] * tanh(|p| / (tau |x'| + 1e-12))
 *   out = active ? cos(angle) x' + sin(angle) |x'| p/max(|p|,1e-20) : x'
 * Math in fp32; x, addend, delta and out share one dtype (bf16 or fp32).
 * The optional addend fuses the HISA low-rank global K/V adapter add
 * (hierarchical_sparse_attn_v18_hisa.py:2579-2591). delta == NULL means no
 * rotation (out = x + addend).
 * ---------------------------------------------------------------------- */
typedef struct {
  int32_t version;
  int32_t dtype;                  /* DWARF_BF16 or DWARF_F32              */
  int64_t B, H, N;
  const void* x;   int64_t sxb, sxh, sxn;
  const void* addend; int64_t sab, sah, san;   /* optional            */
  const void* delta; int64_t sdb, sdh, sdn;
  const float* theta;             /* [H] fp32                             */
  float tau;
  void* out;       int64_t sob, soh, son;
} dwarf_npci_rotate_args;

int dwarf_npci_rotate(const dwarf_npci_rotate_args* args, void* stream);

/* ------------------------------------------------------------------------
 * HISA L3 mixer (production configuration: head_dim 64, chunk 64, selector
 * tile 16, local window 64, top-k <= 4, enumerate_all token selection).
 * ---------------------------------------------------------------------- */

/* Chunk representatives: per 64-token chunk of the global keys,
 * L2-normalise((1-a)*masked mean + a*row of max |k|^2 (first max)), zero for
 * chunks past the valid length, bf16. Replaces
 * _completed_chunk_representatives (hierarchical_sparse_attn_v18_hisa.py:171-219)
 * for representative_mode mean_max_blend (a = blend_alpha; mean: a = 0;
 * max_l2: a = 1). */
typedef struct {
  int32_t version;
  int32_t head_dim, chunk_size;   /* must be 64, 64                       */
  int64_t B, H, T;
  const void* key;                /* bf16 [B, H, T, 64]                   */
  int64_t skb, skh, skn;
  const int32_t* lengths;         /* [B] valid lengths                    */
  float blend_alpha;
  void* reps;                     /* bf16 [B, H, ceil(T/64), 64] contiguous */
  const int64_t* pos;             /* optional device int64 P (decode step):
                                     only chunk P/64 is recomputed        */
} dwarf_hisa_reps_args;

/* Strict-causal top-k tile router: anchor q^ = bf16(normalize(q[16 t])),
 * logits[c] = (q^ . rep_c) / temperature over chunks completed before the
 * tile starts (and inside the valid length); top-k by value, ties to the
 * lower chunk index, -1 where no eligible chunk is left. Replaces forward
 * :2614-2624, _eligibility :222-237 and _build_causal_tile_metadata
 * :290-397 (hierarchical_sparse_attn_v18_hisa.py). ceil(T/64) <= 128. */
typedef struct {
  int32_t version;
  int32_t head_dim, chunk_size, selector_tile;   /* 64, 64, 16            */
  int32_t top_k;
  int64_t B, H, T;
  const void* query;              /* bf16 [B, H, T, 64]                   */
  int64_t sqb, sqh, sqn;
  const void* reps;               /* bf16 [B, H, C, 64]                   */
  const int32_t* lengths;
  float temperature;
  int32_t* top_chunk_idx;         /* [B, H, ceil(T/16), min(top_k, C)]    */
  float* logits;                  /* optional [B, H, tiles, C] (masked)   */
  int64_t tile_begin, tile_count; /* tiles computed (count 0: all from begin;
                                     0, 0 = every tile); decode: one tile */
  const int64_t* pos;             /* optional device int64 P (decode step):
                                     the tile window starts at tile P/16
                                     (tile_begin ignored; tile_count >= 1
                                     tiles), so a captured CUDA graph can
                                     replay at every position             */
} dwarf_hisa_select_args;

/* Route prior of the selected chunks (_selected_route_scores :418-468):
 * route[n, slot] = bf16((q^_n . rep_c - mean over the tile's valid slots) *
 * route_scale[h]), q^_n = bf16(q_n / max(|q_n|, 1e-6)), c the slot's chunk
 * (0 for slots >= k_slots or without a chunk). float32 with sequential sums
 * and no FMA contraction, so it is reproducible bit for bit. */
typedef struct {
  int32_t version;
  int32_t head_dim, selector_tile;  /* 64, 16                             */
  int32_t k_slots;                  /* last dim of top_chunk_idx (<= 4)   */
  int64_t B, H, T, C;
  const void* query;        int64_t sqb, sqh, sqn;
  const void* reps;                 /* bf16 [B, H, C, 64]                 */
  const int32_t* top_chunk_idx;     /* [B, H, tiles, k_slots]             */
  const float* route_scale;         /* [H] = softplus(route_prior_raw)    */
  void* route;                      /* bf16 [B, H, T, 4] contiguous       */
  int64_t tile_begin, tile_count;   /* as dwarf_hisa_select_args          */
  const int64_t* pos;               /* as dwarf_hisa_select_args          */
} dwarf_hisa_route_args;

/* Fused tile attention: for each query n of tile t, one softmax over
 *   local keys  [n-64, n-1] of (local_key, local_value), score q.k/8, and
 *   routed keys of the selected chunks with id < n-64 of (global_key,
 *   global_value), score q.k/8 + route[n, slot] (dwarf_hisa_route).
 * Equals the reference's local lane + global lane + exact LSE merge
 * (:2424-2461, 1002-1100, 808-835). Output bf16, zero past the valid length. */
typedef struct {
  int32_t version;
  int32_t head_dim, chunk_size, selector_tile, local_window;  /* 64,64,16,64 */
  int32_t k_slots;                /* last dim of top_chunk_idx (<= 4)     */
  int64_t B, H, T;
  const void* query;        int64_t sqb, sqh, sqn;
  const void* local_key;    int64_t slkb, slkh, slkn;
  const void* local_value;  int64_t slvb, slvh, slvn;
  const void* global_key;   int64_t sgkb, sgkh, sgkn;
  const void* global_value; int64_t sgvb, sgvh, sgvn;
  const int32_t* top_chunk_idx;   /* [B, H, tiles, k_slots]               */
  const void* route;              /* bf16 [B, H, T, 4] (dwarf_hisa_route) */
  const int32_t* lengths;
  void* out;                int64_t sob, soh, son;   /* bf16              */
  int64_t tile_begin, tile_count; /* as dwarf_hisa_select_args            */
  const int64_t* pos;             /* as dwarf_hisa_select_args            */
  float* lse;                     /* optional fp32 [B, H, T] (contiguous):
                                     row log-sum-exp of the joint softmax in
                                     log2 units (scores x log2 e), +inf for rows
                                     with no key: the input dwarf_hisa_attn_bwd
                                     needs. NULL: not written                */
  int32_t* device_status;         /* optional; set to DWARF_DEVICE_TIMEOUT */
} dwarf_hisa_attn_args;

int dwarf_hisa_reps(const dwarf_hisa_reps_args* args, void* stream);
int dwarf_hisa_select(const dwarf_hisa_select_args* args, void* stream);
int dwarf_hisa_route(const dwarf_hisa_route_args* args, void* stream);
int dwarf_hisa_attn(const dwarf_hisa_attn_args* args, void* stream);

/* Backward of the fused tile attention (dwarf_hisa_attn). Replaces
 * _GlobalHISATritonFn.backward -> _global_lane_backward_kernel
 * (hierarchical_sparse_attn_v18_hisa.py:1982-2027, 1103-1246) together with
 * autograd through the local lane and the LSE merge (:2424-2461, 808-835):
 * with P the joint softmax over the tile's local window and routed chunks,
 * dP = dO . v, delta = dO . O and dS = P (dP - delta):
 *   dq = (1/8) sum dS k,   dk = (1/8) sum dS q,   dv = sum P dO   (local or global K/V),
 *   d_route[n, slot] = sum of dS over the slot's chunk.
 * Three launches on bf16 tensor cores: a query-side kernel (one warp per
 * selector tile: dq, d_route; it writes each row's delta to the caller's
 * scratch plane) and two key-side kernels (64 rows of local / global K/V per
 * CTA: dk, dv). The row lse comes from the forward launch (its lse output). Every output row has exactly one writer: no zero-fill
 * is needed and results are bit-identical between runs. Tensors contiguous,
 * head_dim 64, chunk 64, tile 16, window 64, T <= 8192.
 * ---------------------------------------------------------------------- */
typedef struct {
  int32_t version;
  int32_t k_slots;                /* last dim of top_chunk_idx (<= 4)     */
  int64_t B, H, T;
  const void* query;              /* bf16 [B, H, T, 64]                   */
  const void* local_key;          /* bf16 [B, H, T, 64]                   */
  const void* local_value;
  const void* global_key;
  const void* global_value;
  const int32_t* top_chunk_idx;   /* [B, H, tiles, k_slots]               */
  const void* route;              /* bf16 [B, H, T, 4]                    */
  const int32_t* lengths;         /* [B]                                  */
  const void* out;                /* bf16 [B, H, T, 64] forward output    */
  const void* dout;               /* bf16 [B, H, T, 64]                   */
  float* dq;                      /* [B, H, T, 64] written                */
  float* d_local_key;             /* [B, H, T, 64] written                */
  float* d_local_value;
  float* d_global_key;
  float* d_global_value;
  float* d_route;                 /* [B, H, T, 4] written                 */
  const float* lse;               /* [B, H, T]: the forward's lse output  */
  float* delta;                   /* scratch [B, H, T]: row dO . O        */
} dwarf_hisa_attn_bwd_args;

int dwarf_hisa_attn_bwd(const dwarf_hisa_attn_bwd_args* args, void* stream);

/* ------------------------------------------------------------------------
 * Row-wise block glue (one warp per row of `width` values, width % 256 == 0
 * and <= 1024), with the reference's bf16 rounding points
 * (train/train_dwarf.py:218-240, 260-284, 320-322, 356-364, 439-459).
 * All activations are bf16, rows addressed by an element stride.
 * ---------------------------------------------------------------------- */

/* x_out = bf16(x + bf16(a * bf16(sigmoid(g))))  (gate optional: bf16(x + a);
 * a optional: x_out = x), then n_out = bf16(x_out * rsqrt(mean(x_out^2) +
 * eps) * w). x_out may alias x; x_out NULL skips the write. */
typedef struct {
  int32_t version;
  int32_t w_dtype;                /* DWARF_F32 or DWARF_BF16              */
  int64_t rows, width;
  const void* x;     int64_t sx;
  const void* a;     int64_t sa;  /* optional addend                      */
  const void* g;     int64_t sg;  /* optional gate logits for a           */
  void* x_out;       int64_t sxo; /* optional                             */
  const void* w;                  /* [width] RMSNorm weight               */
  float eps;
  void* n_out;       int64_t sno;
} dwarf_add_rmsnorm_args;

/* x_out = embedding[ids] (bf16), n_out = RMSNorm(x_out) * w. */
typedef struct {
  int32_t version;
  int32_t w_dtype;
  int64_t rows, width, vocab;
  const int64_t* ids;
  const void* embedding;          /* bf16 [vocab, width] contiguous       */
  const void* w;
  float eps;
  void* x_out;                    /* bf16 [rows, width] contiguous        */
  void* n_out;                    /* bf16 [rows, width] contiguous        */
} dwarf_embed_rmsnorm_args;

/* out[r, f] = bf16(bf16(silu(in[r, F + f])) * in[r, f]) -- SwiGLU with the
 * (up | gate) chunk order of SwiGLUFFN (train/train_dwarf.py:230-240). */
typedef struct {
  int32_t version;
  int64_t rows, hidden;           /* hidden = F                            */
  const void* in;    int64_t sin; /* bf16 [rows, 2F]                       */
  void* out;         int64_t sout;/* bf16 [rows, F]                        */
} dwarf_swiglu_args;

/* out = bf16(a * bf16(sigmoid(g))) elementwise over rows. */
typedef struct {
  int32_t version;
  int64_t rows, width;
  const void* a;     int64_t sa;
  const void* g;     int64_t sg;
  void* out;         int64_t so;
} dwarf_gate_mul_args;

/* InterferencePacket epilogue (train/train_dwarf.py:264-276):
 * pooled = bf16 sum_i bf16(mix_i * scan_i) (left to right, bf16 rounding),
 * packet = bf16(dir * tanh(rms / 0.25) * sigmoid(gate_pre)), dir = pooled *
 * rsqrt(mean(pooled^2) + 1e-6), rms = sqrt(mean(pooled^2)). */
typedef struct {
  int32_t version;
  int32_t n_scans;                /* 1..3                                  */
  int64_t rows, width;
  const void* scans[3];  int64_t sscan;   /* bf16 [rows, width] each       */
  float mix[3];                   /* softmax(mix_logits) already in bf16   */
  const void* gate_pre;  int64_t sgp;     /* bf16 gate_proj output          */
  void* out;             int64_t so;
} dwarf_packet_args;

int dwarf_add_rmsnorm(const dwarf_add_rmsnorm_args* args, void* stream);
int dwarf_embed_rmsnorm(const dwarf_embed_rmsnorm_args* args, void* stream);
int dwarf_swiglu(const dwarf_swiglu_args* args, void* stream);
int dwarf_gate_mul(const dwarf_gate_mul_args* args, void* stream);
int dwarf_packet(const dwarf_packet_args* args, void* stream);

/* ------------------------------------------------------------------------
 * bf16 GEMM on the 5th-generation tensor cores (tcgen05, TMA, TMEM) with
 * fused epilogues: out = epilogue(A . B^T), A bf16 [M, K] (row stride lda),
 * B bf16 [N, K] (row stride ldb; a torch Linear weight), fp32 accumulation.
 *
 * Replaces F.linear (+ the following row-wise op) of the reference blocks:
 *   epilogue 0 (DWARF_GEMM_STORE):  out[M, N] = bf16(acc + bias)
 *     -- nn.Linear (train/train_dwarf.py:230-240, 299-322, 325-364, 470);
 *   epilogue 1 (DWARF_GEMM_SWIGLU): out[M, N/2] = SwiGLU of the pair
 *     (up, gate) with dwarf_swiglu's rounding -- SwiGLUFFN.up_gate followed
 *     by silu(gate) * up (train/train_dwarf.py:230-240). B must hold the
 *     up_gate weight in tile-interleaved order: for tile t (of width 2h,
 *     h = swiglu_tile), rows [2ht, 2ht+h) are up rows [ht, ht+h) and rows
 *     [2ht+h, 2h(t+1)) are the matching gate rows (F + ht ...).
 *   epilogue 2 (DWARF_GEMM_RESID_RMSNORM): the residual add and RMSNorm
 *     that follow out_proj / down (train/train_dwarf.py:218-225, 320-322):
 *     v = bf16(resid + bf16(acc)) -> out[M, N] (out may alias resid), and
 *     n_out = bf16((v * rsqrt(mean(v^2) + eps)) * norm_w), as
 *     dwarf_add_rmsnorm rounds them. N must be 256 or 512.
 *   epilogue 3 (DWARF_GEMM_QKVG_PREP): the DSQG qkvg projection (+bias)
 *     with dwarf_dsqg_prep fused in (dsqg_attention_v22.py:3218-3254):
 *     N = 4 D (q | k | v | gate, D = 64 * heads, D % 256 == 0, M = B * T);
 *     q and gate columns go to out (bf16, k/v columns are not written),
 *     y_pre / z_pre come from the bf16 q / k rows and K / V are written
 *     only as the q6 cache (dwarf_q6_pack layout, [B, heads, T] rows).
 *   epilogue 4 (DWARF_GEMM_LSE): lm_head without the logits -- the
 *     forward of LigerFusedLinearCrossEntropyLoss (train/train_dwarf.py:1084,
 *     1134-1138). Per row and 128 columns: (max, sum exp(l - max)) of the
 *     bf16-rounded logits l -> lse_part [M, N/128] float2, (max, index of
 *     its first occurrence) -> arg_part [M, N/128] float2 (index as int bits),
 *     and, with targets [M] int64, target_logit[row] = l[targets[row]].
 *     out is not written (may be NULL); no bias; N % 256 == 0.
 *     dwarf_lse_reduce folds the partials into per-row lse / argmax / loss.
 * Requirements: K % 8 == 0, 16-byte aligned A/B/out and row strides; N a
 * multiple of the tile width (256 or 128 for epilogue 0, 2*swiglu_tile for
 * epilogue 1 with swiglu_tile in {128, 80, 64}).
 * ---------------------------------------------------------------------- */
#define DWARF_GEMM_STORE 0
#define DWARF_GEMM_SWIGLU 1
#define DWARF_GEMM_RESID_RMSNORM 2
#define DWARF_GEMM_QKVG_PREP 3
#define DWARF_GEMM_LSE 4

typedef struct {
  int32_t version;
  int32_t epilogue;               /* DWARF_GEMM_*                          */
  int64_t M, N, K;
  const void* a;     int64_t lda; /* bf16 [M, K]                           */
  const void* b;     int64_t ldb; /* bf16 [N, K]                           */
  const void* bias;               /* optional [N] (epilogue 0)             */
  int32_t bias_dtype;             /* DWARF_F32 or DWARF_BF16               */
  int32_t swiglu_tile;            /* h of epilogue 1                       */
  void* out;         int64_t ldo; /* bf16                                  */
  int32_t* device_status;         /* optional; set to DWARF_DEVICE_TIMEOUT */
  const void* resid; int64_t ldr; /* epilogue 2: bf16 residual [M, N]      */
  const void* norm_w;             /* epilogue 2: [N]                       */
  int32_t norm_w_dtype;           /* DWARF_F32 or DWARF_BF16               */
  float eps;
  void* n_out;       int64_t ldn; /* epilogue 2: bf16 [M, N]               */
  int64_t T;                      /* epilogue 3: rows per batch entry      */
  int32_t heads;                  /* epilogue 3: D / 64                    */
  const float* q_probe;           /* epilogue 3: [4][64] unit probes       */
  const float* k_probe;
  float* y_pre;                   /* epilogue 3: [B, heads, T, 4]          */
  float* z_pre;                   /* epilogue 3: [B, heads, T, 4]          */
  uint8_t* k_codes;               /* epilogue 3: [B, heads, T, 48]         */
  uint16_t* k_scales;             /* epilogue 3: [B, heads, T]             */
  uint8_t* v_codes;
  uint16_t* v_scales;
  int64_t cache_len;              /* epilogue 3: rows per (b, h) of y_pre,
                                     z_pre and the q6 cache (0: T); with the
                                     pointers offset by the first row, a
                                     decode step appends into longer caches */
  void* lse_part;                 /* epilogue 4: float2 [M, N/128]         */
  void* arg_part;                 /* epilogue 4: float2 [M, N/128]         */
  const int64_t* targets;         /* epilogue 4: optional int64 [M]        */
  float* target_logit;            /* epilogue 4: [M] (with targets)        */
  const int64_t* pos;             /* epilogue 3: optional device int64 added
                                     to the first cache row (decode step) */
} dwarf_gemm_args;

int dwarf_gemm_bf16(const dwarf_gemm_args* args, void* stream);

/* Per-row reduction of DWARF_GEMM_LSE partials (parts = N/128 per row):
 * lse[row] = log sum exp over the row's logits, argmax[row] = the first
 * index of its maximum (torch.argmax), and with targets: loss[row] =
 * lse - target_logit (0 where targets[row] == ignore_index), the per-token
 * cross entropy Liger's loss averages (train/train_dwarf.py:1134-1138).
 * Targets outside [0, vocab) other than ignore_index yield loss = NaN. */
typedef struct {
  int32_t version;
  int64_t M, parts, vocab;
  const void* lse_part;           /* float2 [M, parts]                     */
  const void* arg_part;           /* float2 [M, parts]                     */
  const int64_t* targets;         /* optional int64 [M]                    */
  const float* target_logit;      /* [M] (with targets)                    */
  int64_t ignore_index;
  float* lse;                     /* [M]                                   */
  int64_t* argmax;                /* optional [M]                          */
  float* loss;                    /* optional [M] (with targets)           */
} dwarf_lse_reduce_args;

int dwarf_lse_reduce(const dwarf_lse_reduce_args* args, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* DWARF_B200_H */
