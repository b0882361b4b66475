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
This is a forward (inference) engine: a call that would need autograd raises
``NotImplementedError``; CPU tensors raise ``RuntimeError``.
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
            final_state: torch.Tensor | None = None) -> None:
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
    )
    _lib.call("dwarf_ema_scan", args, x.device)


def _forward_only(*tensors: torch.Tensor) -> None:
    if torch.is_grad_enabled() and any(t.requires_grad for t in tensors):
        raise NotImplementedError(
            "dwarf_v2_b200 is a forward (inference) engine; run under torch.no_grad()"
        )


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
    _forward_only(x, ema_factor)
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"causal_ema_scan supports float32/bfloat16 input, got {x.dtype}")
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
    _forward_only(x, alpha)
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"causal_ema_scan supports float32/bfloat16 input, got {x.dtype}")
    alpha32 = alpha.detach().reshape(-1).to(device=x.device, dtype=torch.float32).contiguous()
    out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    _launch(x, out, alpha32, True, False, 0.0, 1.0)
    return out
