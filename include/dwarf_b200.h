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
  DWARF_ERR_VALUE = -9         /* bad scalar argument                         */
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
} dwarf_ema_scan_args;

int64_t dwarf_ema_scan_workspace_bytes(int64_t batch, int64_t seq_len, int64_t width,
                                       int32_t dtype);
int dwarf_ema_scan(const dwarf_ema_scan_args* args, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* DWARF_B200_H */
