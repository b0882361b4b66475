"""q6 KV cache codec (engine-defined format; the reference has no packed KV path).

A row is one (b, h, t) head vector of 64 values:

* ``s = fp16(min(max|x|, 65504))``
* ``c = clamp(rint(x * (31 / float(s))), -31, 31)`` (one IEEE division per row, an fp32
  multiply per value, round half to even; ``s == 0 -> c = 0``)
* 16 groups of 4 codes, each group 3 bytes little-endian of
  ``u0 | u1 << 6 | u2 << 12 | u3 << 18`` with ``u = c & 63``: 48 bytes per row
* dequantisation ``x^ = float(c) * (float(s) / 31)``

``codes`` is ``uint8 [..., 48]`` and ``scales`` is ``float16 [...]``. Packing and
unpacking run as CUDA kernels (``dwarf_q6_pack`` / ``dwarf_q6_unpack``).
"""

from __future__ import annotations

import torch

from . import _lib

ROW_VALUES = 64
ROW_BYTES = 48


def _check_rows(x: torch.Tensor) -> tuple[int, int, int]:
    if x.ndim != 4 or x.shape[-1] != ROW_VALUES:
        raise ValueError(f"expected [B,H,T,64], got {tuple(x.shape)}")
    return x.shape[0], x.shape[1], x.shape[2]


def q6_pack(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Pack ``x[B,H,T,64]`` (bf16 or fp32, last dim contiguous) into (codes, scales)."""
    B, H, T = _check_rows(x)
    _lib.require_cuda(x)
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError(f"q6_pack supports bfloat16/float32, got {x.dtype}")
    if x.stride(-1) != 1:
        x = x.contiguous()
    codes = torch.empty(B, H, T, ROW_BYTES, dtype=torch.uint8, device=x.device)
    scales = torch.empty(B, H, T, dtype=torch.float16, device=x.device)
    args = _lib.Q6PackArgs(
        version=_lib.ABI_VERSION, dtype=_lib.dtype_code(x.dtype), x=x.data_ptr(),
        B=B, H=H, T=T, sxb=x.stride(0), sxh=x.stride(1), sxt=x.stride(2),
        codes=codes.data_ptr(), scb=codes.stride(0), sch=codes.stride(1), sct=codes.stride(2),
        scales=scales.data_ptr(), ssb=scales.stride(0), ssh=scales.stride(1), sst=scales.stride(2),
    )
    _lib.call("dwarf_q6_pack", args, x.device)
    return codes, scales


def q6_unpack(codes: torch.Tensor, scales: torch.Tensor, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Dequantise (codes[B,H,T,48], scales[B,H,T]) to ``dtype`` [B,H,T,64]."""
    if codes.ndim != 4 or codes.shape[-1] != ROW_BYTES or codes.dtype != torch.uint8:
        raise ValueError("codes must be uint8 [B,H,T,48]")
    if scales.shape != codes.shape[:3] or scales.dtype != torch.float16:
        raise ValueError("scales must be float16 [B,H,T]")
    _lib.require_cuda(codes, scales)
    B, H, T = codes.shape[:3]
    out = torch.empty(B, H, T, ROW_VALUES, dtype=dtype, device=codes.device)
    args = _lib.Q6UnpackArgs(
        version=_lib.ABI_VERSION, out_dtype=_lib.dtype_code(dtype), codes=codes.data_ptr(),
        B=B, H=H, T=T, scb=codes.stride(0), sch=codes.stride(1), sct=codes.stride(2),
        scales=scales.data_ptr(), ssb=scales.stride(0), ssh=scales.stride(1), sst=scales.stride(2),
        x=out.data_ptr(), sxb=out.stride(0), sxh=out.stride(1), sxt=out.stride(2),
    )
    _lib.call("dwarf_q6_unpack", args, codes.device)
    return out
