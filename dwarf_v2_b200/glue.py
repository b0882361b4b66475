"""Row-wise block glue kernels (``dwarf_add_rmsnorm``, ``dwarf_embed_rmsnorm``,
``dwarf_swiglu``, ``dwarf_gate_mul``, ``dwarf_packet``).

Each keeps the bf16 rounding points of the reference block code
(train/train_dwarf.py:218-284, 320-322, 356-364, 439-447). Tensors are bf16
with a unit stride on the last dimension; rows are addressed by one stride.
"""

from __future__ import annotations

import torch

from . import _lib


def _rows(t: torch.Tensor) -> tuple[int, int, int]:
    """(rows, width, row_stride) of a [..., width] tensor whose leading dims collapse to one stride."""
    if t.stride(-1) != 1:
        raise ValueError("glue kernels need a unit stride on the last dimension")
    width = t.shape[-1]
    lead, strides = t.shape[:-1], t.stride()[:-1]
    rows = 1
    for n in lead:
        rows *= n
    if not lead:
        return 1, width, width
    for i in range(len(lead) - 1):
        if lead[i] > 1 and strides[i] != strides[i + 1] * lead[i + 1]:
            raise ValueError("glue kernels need rows addressable by a single stride")
    return rows, width, strides[-1]


def _wcode(w: torch.Tensor) -> int:
    if w.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError("norm weight must be bfloat16 or float32")
    return _lib.dtype_code(w.dtype)


def add_rmsnorm(x: torch.Tensor, weight: torch.Tensor, *, addend: torch.Tensor | None = None,
                gate: torch.Tensor | None = None, x_out: torch.Tensor | None = None, eps: float = 1e-6,
                write_sum: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """(x + addend*sigmoid(gate), RMSNorm(that) * weight) with the reference's bf16 rounding."""
    _lib.require_cuda(x, weight, addend, gate)
    rows, width, sx = _rows(x)
    n_out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    weight = weight.contiguous()
    args = _lib.AddRmsNormArgs(version=_lib.ABI_VERSION, w_dtype=_wcode(weight), rows=rows, width=width,
                               x=x.data_ptr(), sx=sx, w=weight.data_ptr(), eps=float(eps),
                               n_out=n_out.data_ptr(), sno=width)
    if addend is not None:
        args.a, args.sa = addend.data_ptr(), _rows(addend)[2]
    if gate is not None:
        args.g, args.sg = gate.data_ptr(), _rows(gate)[2]
    if write_sum and addend is not None:
        if x_out is None:
            x_out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
        args.x_out, args.sxo = x_out.data_ptr(), _rows(x_out)[2]
    _lib.call("dwarf_add_rmsnorm", args, x.device)
    return (x_out if addend is not None else x), n_out


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    return add_rmsnorm(x, weight, eps=eps)[1]


def embed_rmsnorm(ids: torch.Tensor, embedding: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6):
    """(embedding[ids], RMSNorm(embedding[ids]) * weight)."""
    _lib.require_cuda(ids, embedding, weight)
    if embedding.dtype != torch.bfloat16 or not embedding.is_contiguous():
        raise ValueError("embedding must be a contiguous bf16 [vocab, width] table")
    ids64 = ids.to(torch.int64).contiguous()
    vocab, width = embedding.shape
    x = torch.empty(*ids.shape, width, dtype=torch.bfloat16, device=ids.device)
    n = torch.empty_like(x)
    weight = weight.contiguous()
    args = _lib.EmbedRmsNormArgs(version=_lib.ABI_VERSION, w_dtype=_wcode(weight), rows=ids64.numel(),
                                 width=width, vocab=vocab, ids=ids64.data_ptr(), embedding=embedding.data_ptr(),
                                 w=weight.data_ptr(), eps=float(eps), x_out=x.data_ptr(), n_out=n.data_ptr())
    _lib.call("dwarf_embed_rmsnorm", args, ids.device)
    return x, n


def swiglu(up_gate: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _lib.require_cuda(up_gate)
    rows, width, s = _rows(up_gate)
    hidden = width // 2
    if out is None:
        out = torch.empty(*up_gate.shape[:-1], hidden, dtype=torch.bfloat16, device=up_gate.device)
    args = _lib.SwigluArgs(version=_lib.ABI_VERSION, rows=rows, hidden=hidden, in_=up_gate.data_ptr(), sin=s,
                           out=out.data_ptr(), sout=_rows(out)[2])
    _lib.call("dwarf_swiglu", args, up_gate.device)
    return out


def gate_mul(a: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
    _lib.require_cuda(a, g)
    rows, width, sa = _rows(a)
    out = torch.empty(a.shape, dtype=torch.bfloat16, device=a.device)
    args = _lib.GateMulArgs(version=_lib.ABI_VERSION, rows=rows, width=width, a=a.data_ptr(), sa=sa,
                            g=g.data_ptr(), sg=_rows(g)[2], out=out.data_ptr(), so=width)
    _lib.call("dwarf_gate_mul", args, a.device)
    return out


def packet(scans: list[torch.Tensor], mix: list[float], gate_pre: torch.Tensor) -> torch.Tensor:
    _lib.require_cuda(*scans, gate_pre)
    if not 1 <= len(scans) <= 3 or len(mix) != len(scans):
        raise ValueError("packet takes 1..3 scans and one mixture weight per scan")
    rows, width, sscan = _rows(scans[0])
    out = torch.empty(scans[0].shape, dtype=torch.bfloat16, device=gate_pre.device)
    args = _lib.PacketArgs(version=_lib.ABI_VERSION, n_scans=len(scans), rows=rows, width=width,
                           sscan=sscan, gate_pre=gate_pre.data_ptr(), sgp=_rows(gate_pre)[2],
                           out=out.data_ptr(), so=width)
    for i, (sc, w) in enumerate(zip(scans, mix)):
        if _rows(sc)[2] != sscan:
            raise ValueError("all scans must share a row stride")
        args.scans[i] = sc.data_ptr()
        args.mix[i] = float(w)
    _lib.call("dwarf_packet", args, gate_pre.device)
    return out
