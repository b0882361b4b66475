"""NPCI magnitude-aware rotation (``dwarf_npci_rotate``), shared by DSQG and HISA.

Same function as the reference's ``npci_rotate`` (kernels/dsqg_attention_v22.py:223-254)
and ``_magnitude_aware_rotate`` (kernels/hierarchical_sparse_attn_v18_hisa.py:99-125),
in one CUDA kernel. ``addend`` optionally adds a same-shape tensor to ``x`` first
(rounded to ``x``'s dtype), which fuses HISA's low-rank global K/V adapter add.
"""

from __future__ import annotations

import math

import torch

from . import _lib


def npci_rotate_cuda(x: torch.Tensor, x_delta: torch.Tensor | None, theta_h: torch.Tensor, *,
                     strength_tau: float = 0.25, addend: torch.Tensor | None = None,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    tau = float(strength_tau)
    if not math.isfinite(tau) or tau <= 0:
        raise ValueError("strength_tau must be finite and positive")
    if x.ndim != 4 or x.shape[-1] != 64:
        raise ValueError(f"npci rotation expects [B,H,N,64] rows, got {tuple(x.shape)}")
    if (x_delta is not None and x_delta.shape != x.shape) or (addend is not None and addend.shape != x.shape):
        raise ValueError("x, delta (and addend) must share one shape")
    _lib.require_cuda(x, x_delta, theta_h, addend)
    dtype = x.dtype
    if dtype not in (torch.bfloat16, torch.float32):
        raise TypeError(f"npci rotation supports bfloat16/float32, got {dtype}")
    delta = x if x_delta is None else (x_delta if x_delta.dtype == dtype else x_delta.to(dtype))
    if addend is not None and addend.dtype != dtype:
        addend = addend.to(dtype)
    theta = theta_h.detach().reshape(-1).to(device=x.device, dtype=torch.float32).contiguous()
    B, H, N, _ = x.shape
    if theta.numel() != H:
        raise ValueError(f"theta_h must hold {H} per-head angles")
    if out is None:
        out = torch.empty(B, H, N, 64, dtype=dtype, device=x.device)
    args = _lib.NpciArgs(version=_lib.ABI_VERSION, dtype=_lib.dtype_code(dtype), B=B, H=H, N=N,
                         x=x.data_ptr(), sxb=x.stride(0), sxh=x.stride(1), sxn=x.stride(2),
                         delta=delta.data_ptr(), sdb=delta.stride(0), sdh=delta.stride(1), sdn=delta.stride(2),
                         theta=theta.data_ptr(), tau=tau,
                         out=out.data_ptr(), sob=out.stride(0), soh=out.stride(1), son=out.stride(2))
    if addend is not None:
        args.addend, args.sab, args.sah, args.san = addend.data_ptr(), addend.stride(0), addend.stride(1), addend.stride(2)
    if x_delta is None:  # no packet: out = x (+ addend), no rotation
        args.delta = None
    for t in (x, delta, addend, out):
        if t is not None and t.stride(-1) != 1:
            raise ValueError("npci rotation needs a unit stride on the head dimension")
    _lib.call("dwarf_npci_rotate", args, x.device)
    return out


def npci_rotate_autograd(x: torch.Tensor, x_delta: torch.Tensor, theta_h: torch.Tensor, *,
                         strength_tau: float = 0.25) -> torch.Tensor:
    """The same rotation as differentiable elementwise ops on the device, for the
    training path (the reference's ``npci_rotate`` is itself such an op chain,
    kernels/dsqg_attention_v22.py:235-254, differentiated by autograd)."""
    tau = float(strength_tau)
    if not math.isfinite(tau) or tau <= 0:
        raise ValueError("strength_tau must be finite and positive")
    _lib.require_cuda(x, x_delta)
    xf, df = x.float(), x_delta.float()
    theta = theta_h.float().reshape(1, -1, 1, 1)
    norm = xf.norm(dim=-1, keepdim=True).clamp_min(1e-12)
    unit = xf / norm
    perpendicular = df - (df * unit).sum(dim=-1, keepdim=True) * unit
    perpendicular_norm = perpendicular.norm(dim=-1, keepdim=True)
    active = perpendicular_norm > norm * 1e-7
    direction = torch.where(active, perpendicular / perpendicular_norm.clamp_min(1e-20),
                            torch.zeros_like(perpendicular))
    angle = theta * torch.tanh(perpendicular_norm / (tau * norm + 1e-12))
    rotated = torch.cos(angle) * xf + torch.sin(angle) * norm * direction
    return torch.where(active, rotated, xf).to(x.dtype)
