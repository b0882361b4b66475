"""Tensor-core GEMMs with fused epilogues (``dwarf_gemm_bf16``).

Host mirror of the reference's ``F.linear`` calls (train/train_dwarf.py
SwiGLUFFN and the attention projections): ``linear(x, w, bias)`` computes
``x @ w.T + bias`` in bf16 with fp32 accumulation, and ``linear_swiglu``
fuses SwiGLUFFN's ``silu(gate) * up`` into the up_gate projection.
"""

from __future__ import annotations

import torch

from . import _lib

STORE = 0
SWIGLU = 1
RESID_RMSNORM = 2
QKVG_PREP = 3
LSE = 4
SWIGLU_TILES = (128, 80, 64)


def _rows2d(x: torch.Tensor) -> tuple[torch.Tensor, int]:
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    return x2, x2.stride(0)


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 ``x @ weight.T (+ bias)`` on tcgen05; weight [N, K] as nn.Linear stores it."""
    _lib.require_cuda(x, weight, bias)
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise TypeError("linear takes bf16 activations and weights")
    N, K = weight.shape
    x2, lda = _rows2d(x)
    w = weight if weight.stride(-1) == 1 else weight.contiguous()
    M = x2.shape[0]
    if out is None:
        out = torch.empty(*x.shape[:-1], N, dtype=torch.bfloat16, device=x.device)
    o2 = out.view(-1, N)
    args = _lib.GemmArgs(version=_lib.ABI_VERSION, epilogue=STORE, M=M, N=N, K=K, a=x2.data_ptr(), lda=lda,
                         b=w.data_ptr(), ldb=w.stride(0), out=o2.data_ptr(), ldo=o2.stride(0))
    if bias is not None:
        b = bias.contiguous()
        args.bias, args.bias_dtype = b.data_ptr(), _lib.dtype_code(b.dtype)
    _lib.call("dwarf_gemm_bf16", args, x.device)
    return out


def linear_lse(x: torch.Tensor, weight: torch.Tensor, targets: torch.Tensor | None = None, *,
               ignore_index: int = -100):
    """Row-wise logsumexp / argmax (/ cross entropy) of ``x @ weight.T`` without the logits.

    The lm_head GEMM's epilogue reduces each row's bf16-rounded logits per
    128 columns (online max / sum of exp2, first-index argmax, the target's
    logit); ``dwarf_lse_reduce`` folds the partials. Returns (lse fp32 [M],
    argmax int64 [M], loss fp32 [M] or None) over the rows of x; ``loss`` is
    ``lse - logit[target]`` (0 where target == ignore_index).
    """
    _lib.require_cuda(x, weight, targets)
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise TypeError("linear_lse takes bf16 activations and weights")
    N, K = weight.shape
    if N % 256 != 0:
        raise ValueError(f"linear_lse needs a vocabulary that is a multiple of 256, got {N}")
    x2, lda = _rows2d(x)
    w = weight if weight.stride(-1) == 1 else weight.contiguous()
    M = x2.shape[0]
    dev = x.device
    parts = N // 128
    lse_part = torch.empty(M, parts, 2, dtype=torch.float32, device=dev)
    arg_part = torch.empty(M, parts, 2, dtype=torch.float32, device=dev)
    lse = torch.empty(M, dtype=torch.float32, device=dev)
    argmax = torch.empty(M, dtype=torch.int64, device=dev)
    args = _lib.GemmArgs(version=_lib.ABI_VERSION, epilogue=LSE, M=M, N=N, K=K, a=x2.data_ptr(), lda=lda,
                         b=w.data_ptr(), ldb=w.stride(0), lse_part=lse_part.data_ptr(),
                         arg_part=arg_part.data_ptr())
    red = _lib.LseReduceArgs(version=_lib.ABI_VERSION, M=M, parts=parts, vocab=N, lse_part=lse_part.data_ptr(),
                             arg_part=arg_part.data_ptr(), ignore_index=int(ignore_index), lse=lse.data_ptr(),
                             argmax=argmax.data_ptr())
    loss = None
    if targets is not None:
        t = targets.reshape(-1).to(device=dev, dtype=torch.int64).contiguous()
        if t.numel() != M:
            raise ValueError(f"targets must hold one label per row ({M}), got {t.numel()}")
        target_logit = torch.zeros(M, dtype=torch.float32, device=dev)
        loss = torch.empty(M, dtype=torch.float32, device=dev)
        args.targets, args.target_logit = t.data_ptr(), target_logit.data_ptr()
        red.targets, red.target_logit, red.loss = t.data_ptr(), target_logit.data_ptr(), loss.data_ptr()
    if M:
        _lib.call("dwarf_gemm_bf16", args, dev)
        _lib.call("dwarf_lse_reduce", red, dev)
    return lse, argmax, loss


def swiglu_tile(hidden: int) -> int:
    for h in SWIGLU_TILES:
        if hidden % h == 0:
            return h
    raise ValueError(f"no SwiGLU tile width divides hidden={hidden} (supported {SWIGLU_TILES})")


def interleave_up_gate(weight: torch.Tensor, tile: int | None = None) -> torch.Tensor:
    """[2F, K] up_gate weight (up rows then gate rows) -> tile-interleaved rows for linear_swiglu."""
    two_f, K = weight.shape
    F = two_f // 2
    h = tile or swiglu_tile(F)
    up = weight[:F].reshape(F // h, h, K)
    gate = weight[F:].reshape(F // h, h, K)
    return torch.cat([up, gate], dim=1).reshape(two_f, K).contiguous()


def linear_swiglu(x: torch.Tensor, weight_interleaved: torch.Tensor, tile: int,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16(silu(bf16(x @ gate.T)) * bf16(x @ up.T)) with the reference rounding points."""
    _lib.require_cuda(x, weight_interleaved)
    if x.dtype != torch.bfloat16 or weight_interleaved.dtype != torch.bfloat16:
        raise TypeError("linear_swiglu takes bf16 activations and weights")
    N, K = weight_interleaved.shape
    x2, lda = _rows2d(x)
    M = x2.shape[0]
    if out is None:
        out = torch.empty(*x.shape[:-1], N // 2, dtype=torch.bfloat16, device=x.device)
    o2 = out.view(-1, N // 2)
    args = _lib.GemmArgs(version=_lib.ABI_VERSION, epilogue=SWIGLU, M=M, N=N, K=K, a=x2.data_ptr(), lda=lda,
                         b=weight_interleaved.data_ptr(), ldb=weight_interleaved.stride(0), swiglu_tile=tile,
                         out=o2.data_ptr(), ldo=o2.stride(0))
    _lib.call("dwarf_gemm_bf16", args, x.device)
    return out


def linear_add_rmsnorm(x: torch.Tensor, weight: torch.Tensor, resid: torch.Tensor, norm_weight: torch.Tensor,
                       eps: float = 1e-6, x_out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """(v, n): v = bf16(resid + bf16(x @ weight.T)), n = RMSNorm(v) * norm_weight (dwarf_add_rmsnorm rounding).

    Fuses the residual add and the next RMSNorm into the projection (N = 256 or 512);
    ``x_out`` may be ``resid`` itself (in-place residual stream).
    """
    _lib.require_cuda(x, weight, resid, norm_weight)
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16 or resid.dtype != torch.bfloat16:
        raise TypeError("linear_add_rmsnorm takes bf16 activations, weights and residual")
    N, K = weight.shape
    x2, lda = _rows2d(x)
    M = x2.shape[0]
    r2 = resid.reshape(M, N)
    if r2.stride(-1) != 1:
        raise ValueError("resid rows must be contiguous")
    if x_out is None:
        x_out = torch.empty_like(resid)
    n_out = torch.empty_like(resid)
    o2, n2 = x_out.view(M, N), n_out.view(M, N)
    nw = norm_weight.contiguous()
    args = _lib.GemmArgs(version=_lib.ABI_VERSION, epilogue=RESID_RMSNORM, M=M, N=N, K=K, a=x2.data_ptr(),
                         lda=lda, b=weight.data_ptr(), ldb=weight.stride(0), out=o2.data_ptr(), ldo=o2.stride(0),
                         resid=r2.data_ptr(), ldr=r2.stride(0), norm_w=nw.data_ptr(),
                         norm_w_dtype=_lib.dtype_code(nw.dtype), eps=float(eps), n_out=n2.data_ptr(),
                         ldn=n2.stride(0))
    _lib.call("dwarf_gemm_bf16", args, x.device)
    return x_out, n_out


def qkvg_prep(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, heads: int,
              q_probe: torch.Tensor, k_probe: torch.Tensor, *, cache=None, row: int = 0,
              pos: torch.Tensor | None = None):
    """DSQG qkvg projection with the prep pass fused into its epilogue.

    x [B, T, D] bf16; weight [4D, D], bias [4D]. Returns (qkvg, y_pre, z_pre,
    (k_codes, k_scales, v_codes, v_scales)) where qkvg [B, T, 4D] holds valid
    q and gate columns only (K and V exist only as the q6 cache).

    ``cache`` = (y, z, k_codes, k_scales, v_codes, v_scales), contiguous buffers of
    L >= row + T positions per (batch, head) ([B,H,L,4] fp32, [B,H,L,48] u8, [B,H,L]
    fp16): the epilogue writes positions [row, row + T) there instead of allocating
    (the decode cache). The returned tensors are then views of those rows.
    ``pos`` (device int64 [1], with ``cache``) adds a run-time position to ``row``
    (a decode step captured in a CUDA graph); the returned views then start at ``row``.
    """
    _lib.require_cuda(x, weight, bias, q_probe, k_probe)
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise TypeError("qkvg_prep takes bf16 activations and weights")
    B, T, D = x.shape
    N, K = weight.shape
    if N != 4 * D or D != 64 * heads:
        raise ValueError("qkvg_prep expects weight [4D, D] with D = 64 * heads")
    dev = x.device
    x2, lda = _rows2d(x)
    qkvg = torch.empty(B, T, N, dtype=torch.bfloat16, device=dev)
    if cache is None:
        y = torch.empty(B, heads, T, 4, dtype=torch.float32, device=dev)
        z = torch.empty_like(y)
        kc = torch.empty(B, heads, T, 48, dtype=torch.uint8, device=dev)
        vc = torch.empty_like(kc)
        ks = torch.empty(B, heads, T, dtype=torch.float16, device=dev)
        vs = torch.empty_like(ks)
        cache_len = T
    else:
        y, z, kc, ks, vc, vs = cache
        cache_len = y.shape[2]
        shapes = ((y, (B, heads, cache_len, 4), torch.float32), (z, (B, heads, cache_len, 4), torch.float32),
                  (kc, (B, heads, cache_len, 48), torch.uint8), (vc, (B, heads, cache_len, 48), torch.uint8),
                  (ks, (B, heads, cache_len), torch.float16), (vs, (B, heads, cache_len), torch.float16))
        for t, shape, dtype in shapes:
            if tuple(t.shape) != shape or t.dtype != dtype or not t.is_contiguous():
                raise ValueError(f"cache buffer must be contiguous {dtype} {shape}, got {t.dtype} {tuple(t.shape)}")
        if pos is not None and (pos.dtype != torch.int64 or pos.numel() != 1 or not pos.is_cuda):
            raise ValueError("pos must be a one-element int64 CUDA tensor")
        if not 0 <= row <= cache_len - T:
            raise ValueError(f"rows [{row}, {row + T}) exceed the cache length {cache_len}")
        y, z, kc, ks, vc, vs = (t[:, :, row:row + T] for t in (y, z, kc, ks, vc, vs))
    b = bias.contiguous()
    qp, kp = q_probe.float().contiguous(), k_probe.float().contiguous()
    args = _lib.GemmArgs(version=_lib.ABI_VERSION, epilogue=QKVG_PREP, M=B * T, N=N, K=K, a=x2.data_ptr(),
                         lda=lda, b=weight.data_ptr(), ldb=weight.stride(0), bias=b.data_ptr(),
                         bias_dtype=_lib.dtype_code(b.dtype), out=qkvg.data_ptr(), ldo=N, T=T, heads=heads,
                         q_probe=qp.data_ptr(), k_probe=kp.data_ptr(), y_pre=y.data_ptr(), z_pre=z.data_ptr(),
                         k_codes=kc.data_ptr(), k_scales=ks.data_ptr(), v_codes=vc.data_ptr(),
                         v_scales=vs.data_ptr(), cache_len=cache_len,
                         pos=None if pos is None else pos.data_ptr())
    _lib.call("dwarf_gemm_bf16", args, dev)
    return qkvg, y, z, (kc, ks, vc, vs)
