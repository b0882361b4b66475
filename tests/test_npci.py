"""dwarf_npci_rotate against the reference's rotation formula.

The expected values restate the reference's npci_rotate
(kernels/dsqg_attention_v22.py:223-254; the same function as
_magnitude_aware_rotate, kernels/hierarchical_sparse_attn_v18_hisa.py:99-125)
as CPU fp64 torch ops. Both launch shapes are covered: bf16 rows whose starts
are 16-byte aligned (8 lanes per row, 16-byte accesses) and any other layout
(16 lanes per row, element accesses), with and without the fused addend and
with no delta (plain add, no rotation).

Bar: fp32 output within 2e-6 of the fp64 result (relative to the row norm);
bf16 output within one bf16 step (plus the fp32 bar's 2e-6 of the row norm,
which covers outputs near zero where the rotation's two terms cancel) of the
fp64 result rounded to bf16, and equal to it on at least 98% of elements.
"""

import pytest
import torch


def _expected(x, d, theta, tau, addend=None):
    xf = x.double()
    if addend is not None:
        xf = (x + addend).double()  # the add is rounded to x's dtype first
    if d is None:
        return xf
    df = d.double()
    norm = xf.norm(dim=-1, keepdim=True).clamp_min(1e-12)
    unit = xf / norm
    perp = df - (df * unit).sum(-1, keepdim=True) * unit
    pn = perp.norm(dim=-1, keepdim=True)
    active = pn > norm * 1e-7
    direction = torch.where(active, perp / pn.clamp_min(1e-20), torch.zeros_like(perp))
    angle = theta.double().reshape(1, -1, 1, 1) * torch.tanh(pn / (tau * norm + 1e-12))
    return torch.where(active, torch.cos(angle) * xf + torch.sin(angle) * norm * direction, xf)


def _rows(shape, width, seed, dtype, scale=1.0):
    """[B,H,N,64] device rows stored with a row stride of ``width`` elements, and their CPU copy."""
    g = torch.Generator().manual_seed(seed)
    full = (torch.randn(*shape[:-1], width, generator=g) * scale).to(dtype)
    return full.cuda()[..., :64], full[..., :64]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,width", [(torch.bfloat16, 64), (torch.bfloat16, 68), (torch.float32, 64)])
@pytest.mark.parametrize("with_addend", [False, True])
@pytest.mark.parametrize("with_delta", [True, False])
def test_npci_rotate_matches_reference_formula(dtype, width, with_addend, with_delta):
    from dwarf_v2_b200.npci import npci_rotate_cuda

    shape = (2, 3, 301, 64)
    xg, x = _rows(shape, width, 1, dtype)
    dg, d = _rows(shape, width, 2, dtype, 0.3) if with_delta else (None, None)
    ag, a = _rows(shape, width, 3, dtype, 0.1) if with_addend else (None, None)
    if d is not None:
        d[0, 0, :5] = 0.0  # zero delta: inactive rows keep x
        dg[0, 0, :5] = 0.0
    theta = torch.tensor([0.25, -0.1, 0.2])
    out = npci_rotate_cuda(xg, dg, theta.cuda(), strength_tau=0.25, addend=ag).cpu()
    exp = _expected(x, d, theta, 0.25, a)
    if dtype == torch.float32:
        scale = exp.norm(dim=-1, keepdim=True)
        assert float(((out.double() - exp).abs() / scale).max()) <= 2e-6
    else:
        ref = exp.to(torch.bfloat16).double()
        step = ref.abs().clamp_min(2.0 ** -126) * 2.0 ** -7 + 2e-6 * exp.norm(dim=-1, keepdim=True)
        diff = (out.double() - ref).abs()
        assert bool((diff <= step * 1.0001).all()), float((diff / step).max())
        assert float((diff == 0).double().mean()) >= 0.98
