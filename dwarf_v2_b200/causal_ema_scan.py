"""Causal EMA scan on B200: drop-in for the reference ``kernels/causal_ema_scan.py``.

Public surface (same names, argument meaning and errors as the reference):

* ``causal_ema_scan(x, ema_factor, floor=1e-5, ceiling=0.5, *, reset_mask=None)``
  -- ``y[t] = alpha*x[t] + (1-alpha)*y[t-1]`` over ``x[B,N,D]`` with a scalar
  ``alpha = clamp(ema_factor, floor, ceiling)`` (reference :541-567).
* ``bounded_ema_factor`` / ``inverse_bounded_ema_factor`` (reference :37-61).

Extra entry point of this engine:

* ``causal_ema_scan_per_channel(x, alpha)`` -- the same recurrence with one
  unclamped ``alpha`` per channel ``[D]``.

The scan runs as one CUDA launch (``dwarf_ema_scan`` in the C ABI): a chunked
scan chained by decoupled look-back, fp32 state, output in the dtype of ``x``.
Both scans are differentiable (``_CausalEMAFn``, the counterpart of the
reference's ``_CausalEMAFn`` :265-364): the input gradient is the same scan run
over time-reversed ``dy`` (a negative time stride, no copy), and the alpha
gradient is one fused reduction (``dwarf_ema_scan_grad_alpha``). CPU tensors
raise ``RuntimeError``.
"""

from __future__ import annotations

import math

import torch

from . import _lib

__all__ = [
    "bounded_ema_factor",
    "inverse_bounded_ema_factor",
    "causal_ema_scan",
    "causal_ema_scan_per_channel",
]


def bounded_ema_factor(raw: torch.Tensor, *, floor: float = 1e-5, ceiling: float = 0.5) -> torch.Tensor:
    """``floor + (ceiling - floor) * sigmoid(raw)`` (reference causal_ema_scan.py:37-47)."""
    floor, ceiling = float(floor), float(ceiling)
    if not (math.isfinite(floor) and math.isfinite(ceiling) and 0 < floor < ceiling < 1):
        raise ValueError("EMA bounds must satisfy 0 < floor < ceiling < 1")
    return floor + (ceiling - floor) * torch.sigmoid(raw)


def inverse_bounded_ema_factor(alpha: float, *, floor: float = 1e-5, ceiling: float = 0.5) -> float:
    """Raw logit whose bounded factor is ``alpha`` (reference causal_ema_scan.py:50-61)."""
    alpha, floor, ceiling = float(alpha), float(floor), float(ceiling)
    if not floor < alpha < ceiling:
        raise ValueError(f"alpha must be strictly inside ({floor}, {ceiling})")
    p = (alpha - floor) / (ceiling - floor)
    return math.log(p / (1.0 - p))


_workspaces: dict[tuple[int, int], torch.Tensor] = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Look-back scratch per (device, stream), zero-filled once; grows on demand.

    The kernel tags its records with a launch epoch kept in the buffer's
    header, so a buffer is reused across calls without clearing.
    """
    stream = torch.cuda.current_stream(device).cuda_stream
    key = (device.index or 0, stream)
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
        _workspaces[key] = buf
    return buf


def _launch(x: torch.Tensor, out: torch.Tensor, alpha: torch.Tensor, per_channel: bool,
            clamp: bool, floor: float, ceiling: float, init_state: torch.Tensor | None = None,
            final_state: torch.Tensor | None = None, *, wait_limit: int = 0, test_tag_skew: int = 0) -> None:
    lib = _lib.load()
    batch, seq_len, width = x.shape
    code = _lib.dtype_code(x.dtype)
    nbytes = int(lib.dwarf_ema_scan_workspace_bytes(batch, seq_len, width, code))
    if nbytes < 0:
        raise ValueError("unsupported EMA scan shape/dtype")
    ws = _workspace(x.device, nbytes)
    args = _lib.EmaScanArgs(
        version=_lib.ABI_VERSION, dtype=code,
        x=x.data_ptr(), y=out.data_ptr(),
        batch=batch, seq_len=seq_len, width=width,
        sxb=x.stride(0), sxn=x.stride(1), sxd=x.stride(2),
        syb=out.stride(0), syn=out.stride(1), syd=out.stride(2),
        alpha=alpha.data_ptr(), alpha_per_channel=int(per_channel), clamp=int(clamp),
        floor_=floor, ceiling=ceiling,
        workspace=ws.data_ptr(), workspace_bytes=ws.numel(),
        device_status=_lib.device_status_word(x.device).data_ptr(),
        init_state=_lib.ptr(init_state), final_state=_lib.ptr(final_state),
        wait_limit=int(wait_limit), test_tag_skew=int(test_tag_skew),
    )
    _lib.call("dwarf_ema_scan", args, x.device)


def _needs_grad(*tensors: torch.Tensor) -> bool:
    return torch.is_grad_enabled() and any(t.requires_grad for t in tensors)


def _launch_reversed(src: torch.Tensor, dst: torch.Tensor, alpha: torch.Tensor, per_channel: bool) -> None:
    """dst[t] = alpha*src[t] + (1-alpha)*dst[t+1] (dst[T] = 0): the forward scan
    walked from the last token to the first through negative time strides."""
    lib = _lib.load()
    batch, seq_len, width = src.shape
    code = _lib.dtype_code(src.dtype)
    nbytes = int(lib.dwarf_ema_scan_workspace_bytes(batch, seq_len, width, code))
    ws = _workspace(src.device, nbytes)
    last = seq_len - 1
    args = _lib.EmaScanArgs(
        version=_lib.ABI_VERSION, dtype=code,
        x=src.data_ptr() + last * src.stride(1) * src.element_size(),
        y=dst.data_ptr() + last * dst.stride(1) * dst.element_size(),
        batch=batch, seq_len=seq_len, width=width,
        sxb=src.stride(0), sxn=-src.stride(1), sxd=src.stride(2),
        syb=dst.stride(0), syn=-dst.stride(1), syd=dst.stride(2),
        alpha=alpha.data_ptr(), alpha_per_channel=int(per_channel), clamp=0,
        floor_=0.0, ceiling=1.0,
        workspace=ws.data_ptr(), workspace_bytes=ws.numel(),
        device_status=_lib.device_status_word(src.device).data_ptr(),
        init_state=None, final_state=None,
    )
    _lib.call("dwarf_ema_scan", args, src.device)


def _grad_alpha(x: torch.Tensor, y: torch.Tensor, g: torch.Tensor, alpha: torch.Tensor,
                per_channel: bool) -> torch.Tensor:
    """sum over (b, t) of (g / alpha) * (x[t] - y[t-1]) per channel (or in total)."""
    da = torch.empty(x.shape[-1] if per_channel else 1, dtype=torch.float32, device=x.device)
    args = _lib.EmaGradAlphaArgs(
        version=_lib.ABI_VERSION, dtype=_lib.dtype_code(x.dtype),
        x=x.data_ptr(), y=y.data_ptr(), g=g.data_ptr(),
        batch=x.shape[0], seq_len=x.shape[1], width=x.shape[2],
        sxb=x.stride(0), sxn=x.stride(1), sxd=x.stride(2),
        syb=y.stride(0), syn=y.stride(1), syd=y.stride(2),
        sgb=g.stride(0), sgn=g.stride(1), sgd=g.stride(2),
        alpha=alpha.data_ptr(), alpha_per_channel=int(per_channel), pad_=0, da=da.data_ptr(),
    )
    _lib.call("dwarf_ema_scan_grad_alpha", args, x.device)
    return da


class _CausalEMAFn(torch.autograd.Function):
    """Differentiable scan (reference _CausalEMAFn, causal_ema_scan.py:265-364).

    backward: the reverse-time state s[t] = dy[t] + (1-alpha) s[t+1] gives
    dx = alpha * s, which is the forward recurrence run backwards in time over
    dy; d alpha = sum s[t] * (x[t] - y[t-1]). For the scalar API the clamp's
    projected derivative is applied as the reference does (:355-363).
    """

    @staticmethod
    def forward(ctx, x, alpha_input, floor, ceiling, per_channel):
        x = x.contiguous()
        if per_channel:
            alpha = alpha_input.detach().reshape(-1).to(device=x.device, dtype=torch.float32).contiguous()
        else:
            alpha = alpha_input.detach().reshape(1).to(device=x.device, dtype=torch.float32)
            alpha = alpha.clamp(float(floor), float(ceiling))
        out = torch.empty_like(x)
        _launch(x, out, alpha, per_channel, False, 0.0, 1.0)
        ctx.save_for_backward(x, out, alpha_input, alpha)
        ctx.floor, ctx.ceiling, ctx.per_channel = float(floor), float(ceiling), bool(per_channel)
        return out

    @staticmethod
    def backward(ctx, dy):
        x, y, alpha_input, alpha = ctx.saved_tensors
        dy = dy.contiguous()
        need_da = bool(ctx.needs_input_grad[1])
        if need_da and dy.dtype != torch.float32:
            g = torch.empty(dy.shape, dtype=torch.float32, device=dy.device)
            _launch_reversed(dy.float(), g, alpha, ctx.per_channel)
            dx = g.to(dy.dtype)
        else:
            dx = torch.empty_like(dy)
            _launch_reversed(dy, dx, alpha, ctx.per_channel)
            g = dx
        if not need_da:
            return dx, None, None, None, None
        da = _grad_alpha(x, y, g, alpha, ctx.per_channel)
        da = da.reshape_as(alpha_input).to(alpha_input.dtype)
        if not ctx.per_channel:
            blocked = ((alpha_input <= ctx.floor) & (da > 0)) | ((alpha_input >= ctx.ceiling) & (da < 0))
            da = torch.where(blocked, torch.zeros_like(da), da)
        return dx, da, None, None, None


def causal_ema_scan(
    x: torch.Tensor,
    ema_factor: torch.Tensor,
    floor: float = 1e-5,
    ceiling: float = 0.5,
    *,
    reset_mask: torch.Tensor | None = None,
    initial_state: torch.Tensor | None = None,
    return_final_state: bool = False,
):
    """Scalar-alpha causal EMA over ``x[B,N,D]`` (reference causal_ema_scan.py:541-567).

    Engine extensions for incremental decoding: ``initial_state`` (fp32 [B, D]) is
    y[-1] instead of zero, and ``return_final_state`` also returns the fp32 state
    after the last token (the state a continuation starts from).
    """
    if x.ndim != 3:
        raise ValueError(f"x must be [B,N,D], got {tuple(x.shape)}")
    if ema_factor.numel() != 1:
        raise ValueError("ema_factor must contain one scalar")
    if not (0 < float(floor) < float(ceiling) < 1):
        raise ValueError("EMA bounds must satisfy 0 < floor < ceiling < 1")
    if reset_mask is not None:
        raise NotImplementedError("reset-aware EMA is not part of the prefill engine")
    _lib.require_cuda(x)
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"causal_ema_scan supports float32/bfloat16 input, got {x.dtype}")
    if _needs_grad(x, ema_factor):
        if initial_state is not None or return_final_state:
            raise NotImplementedError("initial_state / return_final_state are inference-only")
        return _CausalEMAFn.apply(x, ema_factor, float(floor), float(ceiling), False)
    alpha = ema_factor.detach().reshape(1).to(device=x.device, dtype=torch.float32)
    out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    B, _, D = x.shape
    if initial_state is not None:
        if initial_state.shape != (B, D) or initial_state.dtype != torch.float32:
            raise ValueError("initial_state must be float32 [B, D]")
        _lib.require_cuda(initial_state)
        initial_state = initial_state.contiguous()
    final = torch.empty(B, D, dtype=torch.float32, device=x.device) if return_final_state else None
    _launch(x, out, alpha, False, True, float(floor), float(ceiling), initial_state, final)
    return (out, final) if return_final_state else out


def causal_ema_scan_per_channel(x: torch.Tensor, alpha: torch.Tensor) -> torch.Tensor:
    """``y[t,d] = alpha[d]*x[t,d] + (1-alpha[d])*y[t-1,d]`` with no clamping.

    A decay written as ``y_t = a*y_{t-1} + (1-a)*x_t`` maps to ``alpha = 1 - a``.
    """
    if x.ndim != 3:
        raise ValueError(f"x must be [B,N,D], got {tuple(x.shape)}")
    if alpha.numel() != x.shape[-1]:
        raise ValueError(f"alpha must have {x.shape[-1]} entries, got {alpha.numel()}")
    _lib.require_cuda(x)
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"causal_ema_scan supports float32/bfloat16 input, got {x.dtype}")
    if _needs_grad(x, alpha):
        return _CausalEMAFn.apply(x, alpha, 0.0, 1.0, True)
    alpha32 = alpha.detach().reshape(-1).to(device=x.device, dtype=torch.float32).contiguous()
    out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    _launch(x, out, alpha32, True, False, 0.0, 1.0)
    return out
