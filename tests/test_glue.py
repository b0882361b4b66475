"""The row-wise glue kernels against the reference's own formulas.

Each kernel (dwarf_add_rmsnorm, dwarf_embed_rmsnorm, dwarf_swiglu,
dwarf_gate_mul, dwarf_packet) runs on the GPU through the C ABI; the expected
values are the reference's block code restated as CPU torch ops in its own
order and dtypes (train/train_dwarf.py:218-227 RMSNorm, :230-240 SwiGLU,
:260-284 InterferencePacket, :320-322 and :356-364 residual adds, :439-447
embedding; the HISA output gate W_o(o) * sigmoid(gate),
kernels/hierarchical_sparse_attn_v18_hisa.py:2777). CPU bf16 tensor ops round
every intermediate to bf16 exactly where the reference's CUDA ops do.

Bar: residual sums (bf16(x + a)) bit-exact; normalised / activated outputs
within one bf16 step of the reference everywhere and bit-exact on at least 99%
of elements (the remaining flips come from fp32 summation order and the
device's rsqrt/exp approximations; a misplaced rounding point moves far more
elements).
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F


def _ref_rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """train/train_dwarf.py:224-227."""
    xf = x.float()
    normalized = xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps)
    return (normalized * w.float()).to(x.dtype)


def _close_bf16(out: torch.Tensor, ref: torch.Tensor, exact_frac: float = 0.99) -> None:
    a, b = out.float().cpu(), ref.float().cpu()
    step = b.abs().clamp_min(2.0 ** -126) * 2.0 ** -7  # one bf16 ulp (8 significant bits) at ref
    diff = (a - b).abs()
    assert bool((diff <= step * 1.0001).all()), float((diff / step).max())
    frac = float((diff == 0).double().mean())
    assert frac >= exact_frac, frac


def _inputs(rows: int, width: int, seed: int, scale: float = 1.0):
    g = torch.Generator().manual_seed(seed)
    return lambda s=scale: (torch.randn(rows, width, generator=g) * s).to(torch.bfloat16)


@pytest.mark.gpu
@pytest.mark.parametrize("width,w_dtype", [(512, torch.float32), (512, torch.bfloat16), (768, torch.float32)])
def test_add_rmsnorm_matches_reference_residual_add_and_rmsnorm(width, w_dtype):
    """DSQGBlock.forward (:320-322): x = x + attn(norm1(x)); norm2(x)."""
    from dwarf_v2_b200 import glue

    r = _inputs(300, width, seed=width)
    x, a = r(0.3), r(0.1)
    w = (1.0 + 0.1 * torch.randn(width, generator=torch.Generator().manual_seed(1))).to(w_dtype)
    x_sum, n = glue.add_rmsnorm(x.cuda(), w.cuda(), addend=a.cuda())
    ref_sum = x + a
    assert torch.equal(x_sum.cpu(), ref_sum)
    _close_bf16(n, _ref_rmsnorm(ref_sum, w))
    n_only = glue.rmsnorm(x.cuda(), w.cuda())
    _close_bf16(n_only, _ref_rmsnorm(x, w))


@pytest.mark.gpu
def test_add_rmsnorm_gated_matches_reference_hisa_residual():
    """GlobalMixerBlock.forward (:356-364) with the HISA output gate: x = x + W_o(o) * sigmoid(gate)."""
    from dwarf_v2_b200 import glue

    r = _inputs(257, 512, seed=7)
    x, proj, gate = r(0.3), r(0.1), r(2.0)
    w = (1.0 + 0.1 * torch.randn(512, generator=torch.Generator().manual_seed(2)))
    x_sum, n = glue.add_rmsnorm(x.cuda(), w.cuda(), addend=proj.cuda(), gate=gate.cuda())
    ref_sum = x + proj * torch.sigmoid(gate)
    assert torch.equal(x_sum.cpu(), ref_sum)
    _close_bf16(n, _ref_rmsnorm(ref_sum, w))


@pytest.mark.gpu
def test_embed_rmsnorm_matches_reference_embedding_and_first_norm():
    """forward_hidden (:439-447): x = embedding(ids) (bf16 on CUDA), then block 0's norm1."""
    from dwarf_v2_b200 import glue

    g = torch.Generator().manual_seed(3)
    emb = (torch.randn(1000, 512, generator=g) * 0.02).to(torch.bfloat16)
    ids = torch.randint(0, 1000, (3, 171), generator=g)
    w = 1.0 + 0.1 * torch.randn(512, generator=g)
    x, n = glue.embed_rmsnorm(ids.cuda(), emb.cuda(), w.cuda())
    assert torch.equal(x.cpu(), emb[ids])
    _close_bf16(n, _ref_rmsnorm(emb[ids], w))


@pytest.mark.gpu
def test_swiglu_matches_reference():
    """SwiGLUFFN.forward (:239-240): up, gate = up_gate(x).chunk(2); silu(gate) * up."""
    from dwarf_v2_b200 import glue

    g = torch.Generator().manual_seed(4)
    up_gate = (torch.randn(333, 2 * 1600, generator=g) * 1.5).to(torch.bfloat16)
    out = glue.swiglu(up_gate.cuda())
    up, gate = up_gate.chunk(2, dim=-1)
    _close_bf16(out, F.silu(gate) * up)


@pytest.mark.gpu
def test_gate_mul_matches_reference():
    """The HISA output gate (hierarchical_sparse_attn_v18_hisa.py:2777): a * sigmoid(g) in bf16."""
    from dwarf_v2_b200 import glue

    r = _inputs(211, 512, seed=5)
    a, gt = r(0.5), r(3.0)
    _close_bf16(glue.gate_mul(a.cuda(), gt.cuda()), a * torch.sigmoid(gt))


@pytest.mark.gpu
def test_packet_matches_reference_interference_packet():
    """InterferencePacket.forward (:260-280) after the scans: bf16 mixture of the three
    scans, RMS direction, tanh confidence, fp32 sigmoid gate, one rounding to bf16."""
    from dwarf_v2_b200 import glue

    g = torch.Generator().manual_seed(6)
    rows, width = 300, 512
    scans = [(torch.randn(rows, width, generator=g) * s).to(torch.bfloat16) for s in (0.05, 0.1, 0.3)]
    gate_pre = (torch.randn(rows, width, generator=g) * 2.0 - 2.0).to(torch.bfloat16)
    mix_logits = torch.randn(3, generator=g)
    mixture = torch.softmax(mix_logits.float(), dim=0)
    pooled = sum(weight.to(scans[0].dtype) * scan for weight, scan in zip(mixture, scans, strict=True))
    pooled_float = pooled.float()
    rms = pooled_float.square().mean(-1, keepdim=True).sqrt()
    direction = pooled_float * torch.rsqrt(pooled_float.square().mean(-1, keepdim=True) + 1e-6)
    confidence = torch.tanh(rms / 0.25)
    gate = torch.sigmoid(gate_pre.float())
    ref = (direction * confidence * gate).to(torch.bfloat16)
    out = glue.packet([s.cuda() for s in scans], mixture.to(torch.bfloat16).float().tolist(), gate_pre.cuda())
    _close_bf16(out, ref)
