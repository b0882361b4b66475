"""Causal EMA scan backward: the oracle's gradients pinned to golden vectors made
by autograd through the reference's ``_reference`` (CPU), and the engine's
autograd path (reverse-time ``dwarf_ema_scan`` + ``dwarf_ema_scan_grad_alpha``
through the C ABI) checked against the oracle (GPU).

Tolerances: dx 1e-5 max-abs for fp32 (the fp32 EMA tolerance of the north-star
spec); d alpha, a sum over up to 16.7 M products, 1e-4 relative to the largest
|d alpha| (fp32 atomics in an unspecified order).
"""

import numpy as np
import pytest
import torch

from oracle import ema as oracle_ema
from tests._golden import load

FIXTURES = [("ema_bwd_scalar_f64", False), ("ema_bwd_scalar_f32", False), ("ema_bwd_per_channel_f32", True)]


@pytest.mark.parametrize("name,per_channel", FIXTURES)
def test_oracle_backward_matches_reference_autograd(name, per_channel):
    g = load(name)
    dx, da = oracle_ema.ema_scan_backward(g["x"].numpy(), g["y"].numpy(), g["dy"].numpy(),
                                          g["alpha"].double().numpy(), per_channel=per_channel)
    assert np.abs(dx - g["dx"].double().numpy()).max() < 1e-5
    ref_da = g["da"].double().numpy().reshape(-1)
    assert np.abs(np.reshape(da, -1) - ref_da).max() <= 1e-5 * max(1.0, np.abs(ref_da).max())


def _check(dx, da, ref_dx, ref_da, dx_tol=1e-5):
    assert np.abs(dx.detach().double().cpu().numpy() - ref_dx).max() < dx_tol
    ref_da = np.reshape(ref_da, -1)
    got = da.detach().double().cpu().numpy().reshape(-1)
    assert np.abs(got - ref_da).max() <= 1e-4 * max(1.0, np.abs(ref_da).max())


@pytest.mark.gpu
@pytest.mark.parametrize("name,per_channel", FIXTURES[1:])
def test_autograd_matches_reference_golden(name, per_channel):
    from dwarf_v2_b200.causal_ema_scan import causal_ema_scan, causal_ema_scan_per_channel

    g = load(name)
    x = g["x"].float().cuda().requires_grad_(True)
    alpha = g["alpha"].float().cuda().requires_grad_(True)
    y = causal_ema_scan_per_channel(x, alpha) if per_channel else causal_ema_scan(x, alpha)
    y.backward(g["dy"].float().cuda())
    _check(x.grad, alpha.grad, g["dx"].double().numpy(), g["da"].double().numpy())


@pytest.mark.gpu
def test_autograd_config2_full_size():
    """BASELINE config 2 at full size (B=16, T=2048, D=512 fp32, a = sigmoid(N(0,1)))
    with a random upstream gradient, against the oracle's backward."""
    from dwarf_v2_b200.causal_ema_scan import causal_ema_scan_per_channel

    g = torch.Generator().manual_seed(0)
    x = torch.randn(16, 2048, 512, generator=g)
    alpha = 1.0 - torch.sigmoid(torch.randn(512, generator=g))
    dy = torch.randn(16, 2048, 512, generator=g)
    xc = x.cuda().requires_grad_(True)
    ac = alpha.cuda().requires_grad_(True)
    y = causal_ema_scan_per_channel(xc, ac)
    y.backward(dy.cuda())
    ref_y = oracle_ema.ema_scan(x.numpy(), alpha.double().numpy())
    ref_dx, ref_da = oracle_ema.ema_scan_backward(x.numpy(), ref_y, dy.numpy(), alpha.double().numpy(),
                                                  per_channel=True)
    _check(xc.grad, ac.grad, ref_dx, ref_da)
    from dwarf_v2_b200 import _lib

    assert _lib.read_and_clear_device_status(torch.device("cuda:0")) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(1, 1, 8), (2, 33, 40), (2, 50, 13), (3, 517, 264)])
def test_autograd_bf16_and_ragged(shape):
    """bf16 activations as the model feeds the scan; ragged T and D. dx is stored
    in bf16 (one rounding of the fp32 state), d alpha from the fp32 state."""
    from dwarf_v2_b200.causal_ema_scan import causal_ema_scan

    g = torch.Generator().manual_seed(sum(shape))
    x = torch.randn(*shape, generator=g).to(torch.bfloat16)
    dy = torch.randn(*shape, generator=g).to(torch.bfloat16)
    xc = x.cuda().requires_grad_(True)
    a = torch.tensor([1.0 / 16.0], device="cuda", requires_grad=True)
    y = causal_ema_scan(xc, a)
    y.backward(dy.cuda())
    assert xc.grad.dtype == torch.bfloat16
    ref_dx, ref_da = oracle_ema.ema_scan_backward(x.float().numpy(), y.detach().float().cpu().numpy(),
                                                  dy.float().numpy(), np.array([1.0 / 16.0]))
    assert np.abs(xc.grad.double().cpu().numpy() - ref_dx).max() <= 2 ** -7 * max(1.0, np.abs(ref_dx).max())
    assert abs(float(a.grad) - float(ref_da)) <= 1e-4 * max(1.0, abs(float(ref_da)))


@pytest.mark.gpu
def test_projected_clamp_derivative():
    """alpha_input at/above the ceiling: d alpha is zeroed when it points outward
    (reference causal_ema_scan.py:355-363), kept when it points inward."""
    from dwarf_v2_b200.causal_ema_scan import causal_ema_scan

    g = torch.Generator().manual_seed(9)
    x = torch.randn(2, 64, 32, generator=g).cuda()
    for sign in (1.0, -1.0):
        a = torch.tensor([0.7], device="cuda", requires_grad=True)
        y = causal_ema_scan(x, a)
        dy = sign * x  # pushes d alpha to one sign or the other
        y.backward(dy)
        ref_y = oracle_ema.ema_scan(x.cpu().numpy(), np.array([0.5]))
        _, ref_da = oracle_ema.ema_scan_backward(x.cpu().numpy(), ref_y, dy.cpu().numpy(), np.array([0.5]))
        expected = 0.0 if ref_da < 0 else ref_da
        assert abs(float(a.grad) - expected) <= 1e-4 * max(1.0, abs(ref_da))
