"""Causal EMA scan: oracle pinned to the reference's golden vectors (CPU) and the
CUDA kernel (dwarf_ema_scan through the C ABI) checked against the oracle (GPU).

Tolerances: fp32/fp64 inputs 1e-5 max-abs (the fp32 EMA tolerance of the
north-star spec); bf16 outputs within one bf16 rounding step (2**-7 relative),
since kernel and reference round differently-ordered fp32 states.
"""

import numpy as np
import pytest
import torch

from oracle import ema as oracle_ema
from tests._golden import load

FIXTURES = ["ema_reference_main_f64", "ema_scalar_clamped_f32", "ema_scalar_bf16"]


@pytest.mark.parametrize("name", FIXTURES)
def test_oracle_matches_reference_golden(name):
    g = load(name)
    y = oracle_ema.ema_scan(g["x"].float().numpy() if g["x"].dtype == torch.bfloat16 else g["x"].numpy(),
                            g["alpha"].double().numpy(), clamp=(1e-5, 0.5))
    ref = g["y"].double().numpy()
    if g["y"].dtype == torch.bfloat16:
        y = torch.from_numpy(y).float().to(torch.bfloat16).double().numpy()
        assert np.abs(y - ref).max() <= 2 ** -7 * max(1.0, np.abs(ref).max())
    else:
        assert np.abs(y - ref).max() < 1e-6


def test_oracle_per_channel_matches_reference_golden():
    g = load("ema_per_channel_f32")
    y = oracle_ema.ema_scan_decay_form(g["x"].numpy(), g["decay"].numpy())
    assert np.abs(y - g["y"].double().numpy()).max() < 1e-5


def test_bounded_factor_roundtrip():
    from dwarf_v2_b200.causal_ema_scan import bounded_ema_factor, inverse_bounded_ema_factor

    for a in (1 / 16, 1 / 64, 1 / 256, 0.3):
        raw = inverse_bounded_ema_factor(a)
        assert abs(float(bounded_ema_factor(torch.tensor(raw, dtype=torch.float64))) - a) < 1e-12
    with pytest.raises(ValueError):
        inverse_bounded_ema_factor(0.7)
    with pytest.raises(ValueError):
        bounded_ema_factor(torch.zeros(1), floor=0.6, ceiling=0.5)


def test_api_errors_without_gpu():
    from dwarf_v2_b200.causal_ema_scan import causal_ema_scan

    with pytest.raises(ValueError):
        causal_ema_scan(torch.zeros(2, 3), torch.tensor([0.1]))
    with pytest.raises(ValueError):
        causal_ema_scan(torch.zeros(2, 3, 4), torch.tensor([0.1, 0.2]))
    with pytest.raises(ValueError):
        causal_ema_scan(torch.zeros(2, 3, 4), torch.tensor([0.1]), floor=0.6, ceiling=0.5)
    with pytest.raises(RuntimeError):  # CPU tensors: no fallback
        causal_ema_scan(torch.zeros(2, 3, 4), torch.tensor([0.1]))


# ----------------------------------------------------------------- GPU parity

def _tol_check(y_gpu: torch.Tensor, ref: np.ndarray, dtype: torch.dtype):
    y = y_gpu.double().cpu().numpy()
    if dtype == torch.bfloat16:
        scale = np.maximum(np.abs(ref), 1e-3)
        rel = np.abs(y - ref) / scale
        assert rel.max() <= 2 ** -7, rel.max()
    else:
        assert np.abs(y - ref).max() < 1e-5, np.abs(y - ref).max()


@pytest.mark.gpu
@pytest.mark.parametrize("name", FIXTURES)
def test_kernel_matches_reference_golden(name):
    from dwarf_v2_b200.causal_ema_scan import causal_ema_scan

    g = load(name)
    x = g["x"]
    if x.dtype == torch.float64:
        x = x.float()
    y = causal_ema_scan(x.cuda(), g["alpha"].float().cuda())
    torch.cuda.synchronize()
    ref = oracle_ema.ema_scan(x.float().numpy(), g["alpha"].double().numpy(), clamp=(1e-5, 0.5))
    _tol_check(y, ref, x.dtype)
    gold = g["y"].double().numpy()
    tol = 2 ** -7 if x.dtype == torch.bfloat16 else 1e-5
    assert np.abs(y.double().cpu().numpy() - gold).max() <= tol * max(1.0, np.abs(gold).max())


@pytest.mark.gpu
@pytest.mark.parametrize(
    "shape,dtype,strided",
    [
        ((1, 1, 1), torch.float32, False),
        ((2, 9, 7), torch.float32, False),
        ((3, 1000, 96), torch.float32, False),
        ((2, 777, 513), torch.float32, False),
        ((4, 2048, 512), torch.float32, False),
        ((2, 2048, 512), torch.bfloat16, False),
        ((3, 517, 264), torch.bfloat16, False),
        ((2, 300, 128), torch.float32, True),
        ((2, 300, 128), torch.bfloat16, True),
    ],
)
def test_kernel_per_channel_shapes(shape, dtype, strided):
    from dwarf_v2_b200.causal_ema_scan import causal_ema_scan_per_channel

    g = torch.Generator().manual_seed(sum(shape))
    B, N, D = shape
    if strided:
        base = torch.randn(B, N, 2 * D, generator=g).to(dtype)
        x = base[:, :, ::2]
    else:
        x = torch.randn(B, N, D, generator=g).to(dtype)
    decay = torch.sigmoid(torch.randn(D, generator=g))
    y = causal_ema_scan_per_channel(x.cuda(), (1.0 - decay).cuda())
    torch.cuda.synchronize()
    ref = oracle_ema.ema_scan_decay_form(x.float().numpy(), decay.double().numpy())
    _tol_check(y, ref, dtype)


@pytest.mark.gpu
@pytest.mark.parametrize(
    "shape,dtype,per_channel",
    [
        ((160, 300, 32), torch.float32, True),     # one 32-channel block per row, a partial chunk
        ((150, 1000, 96), torch.float32, False),   # scalar alpha, three blocks per row
        ((40, 517, 264), torch.bfloat16, True),    # a 16-byte width edge (8 of 64 channels)
        ((160, 2048, 512), torch.bfloat16, False),  # the model's packet scan at 160 rows
    ],
)
def test_kernel_many_series_shapes(shape, dtype, per_channel):
    """Many independent (row, channel block) series with partial last tiles, a 16-byte
    width edge and both alpha forms, against the oracle."""
    from dwarf_v2_b200.causal_ema_scan import causal_ema_scan, causal_ema_scan_per_channel

    g = torch.Generator().manual_seed(sum(shape))
    B, N, D = shape
    x = torch.randn(B, N, D, generator=g).to(dtype)
    if per_channel:
        decay = torch.sigmoid(torch.randn(D, generator=g))
        y = causal_ema_scan_per_channel(x.cuda(), (1.0 - decay).cuda())
        ref = oracle_ema.ema_scan_decay_form(x.float().numpy(), decay.double().numpy())
    else:
        alpha = torch.tensor([0.03])
        y = causal_ema_scan(x.cuda(), alpha.cuda())
        ref = oracle_ema.ema_scan(x.float().numpy(), alpha.double().numpy(), clamp=(1e-5, 0.5))
    torch.cuda.synchronize()
    _tol_check(y, ref, dtype)


@pytest.mark.gpu
@pytest.mark.parametrize("split", [1, 300, 1499])
def test_kernel_many_series_continuation(split):
    """initial_state/final_state with many series in flight (160 rows x 256 channels)."""
    from dwarf_v2_b200.causal_ema_scan import causal_ema_scan

    g = torch.Generator().manual_seed(9)
    x = torch.randn(160, 1500, 256, generator=g).cuda()
    a = torch.tensor([0.07], device="cuda")
    full, full_state = causal_ema_scan(x, a, return_final_state=True)
    head, state = causal_ema_scan(x[:, :split].contiguous(), a, return_final_state=True)
    tail, end_state = causal_ema_scan(x[:, split:].contiguous(), a, initial_state=state,
                                      return_final_state=True)
    torch.testing.assert_close(state, full[:, split - 1].float(), atol=1e-6, rtol=0)
    torch.testing.assert_close(torch.cat([head, tail], 1), full, atol=1e-5, rtol=0)
    torch.testing.assert_close(end_state, full_state, atol=1e-5, rtol=0)


@pytest.mark.gpu
def test_kernel_config2_full_size_properties():
    """BASELINE config 2 at full size: B=16, T=2048, D=512 fp32, a = sigmoid(N(0,1))."""
    from dwarf_v2_b200.causal_ema_scan import causal_ema_scan_per_channel

    g = torch.Generator().manual_seed(0)
    x = torch.randn(16, 2048, 512, generator=g)
    decay = torch.sigmoid(torch.randn(512, generator=g))
    y = causal_ema_scan_per_channel(x.cuda(), (1.0 - decay).cuda()).cpu()
    ref = oracle_ema.ema_scan_decay_form(x.numpy(), decay.double().numpy())
    assert np.abs(y.double().numpy() - ref).max() < 1e-5
    # linearity: scan(2x + 3) == 2 scan(x) + scan(3)
    y2 = causal_ema_scan_per_channel((2 * x + 3).cuda(), (1.0 - decay).cuda()).cpu()
    y3 = causal_ema_scan_per_channel(torch.full_like(x, 3.0).cuda(), (1.0 - decay).cuda()).cpu()
    assert (y2 - (2 * y + y3)).abs().max() < 1e-4
    from dwarf_v2_b200 import _lib

    assert _lib.read_and_clear_device_status(torch.device("cuda:0")) == 0


@pytest.mark.gpu
def test_kernel_causality_and_repeatability():
    from dwarf_v2_b200.causal_ema_scan import causal_ema_scan

    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 1500, 256, generator=g).cuda()
    a = torch.tensor([0.05], device="cuda")
    y1 = causal_ema_scan(x, a)
    x2 = x.clone()
    x2[:, 700:] += 10.0
    y2 = causal_ema_scan(x2, a)
    assert torch.equal(y1[:, :700], y2[:, :700])
    assert torch.equal(y1, causal_ema_scan(x, a))


@pytest.mark.gpu
@pytest.mark.parametrize("split", [1, 37, 1024, 1499])
def test_kernel_continuation_matches_one_pass(split):
    """initial_state/final_state: scanning [0,split) then [split,N) from the carried
    state reproduces the single pass (the decode path's EMA continuation)."""
    from dwarf_v2_b200.causal_ema_scan import causal_ema_scan

    g = torch.Generator().manual_seed(5)
    x = torch.randn(2, 1500, 256, generator=g).cuda()
    a = torch.tensor([0.07], device="cuda")
    full, full_state = causal_ema_scan(x, a, return_final_state=True)
    head, state = causal_ema_scan(x[:, :split].contiguous(), a, return_final_state=True)
    tail, end_state = causal_ema_scan(x[:, split:].contiguous(), a, initial_state=state,
                                      return_final_state=True)
    torch.testing.assert_close(state, full[:, split - 1].float(), atol=1e-6, rtol=0)
    torch.testing.assert_close(torch.cat([head, tail], 1), full, atol=1e-5, rtol=0)
    torch.testing.assert_close(end_state, full_state, atol=1e-5, rtol=0)


@pytest.mark.gpu
def test_lookback_wait_runs_out_reports_timeout_and_context_stays_usable():
    """Bounded-wait path without a fault: with test_tag_skew the look-back waits for
    records that no writer produces, gives up after the host-set poll limit and records
    DWARF_DEVICE_TIMEOUT in the status word; check_device_status raises and clears it,
    and the next scan on the same context is exact."""
    from dwarf_v2_b200 import _lib, check_device_status
    from dwarf_v2_b200.causal_ema_scan import _launch, causal_ema_scan_per_channel

    g = torch.Generator().manual_seed(11)
    x = torch.randn(2, 1024, 256, generator=g).cuda()
    alpha = torch.rand(256, generator=g).cuda()
    check_device_status(x.device)  # a clean start
    out = torch.empty_like(x)
    _launch(x, out, alpha, True, False, 0.0, 1.0, wait_limit=64, test_tag_skew=1)
    with pytest.raises(_lib.DeviceTimeoutError):
        check_device_status(x.device)
    y = causal_ema_scan_per_channel(x, alpha).cpu()
    ref = oracle_ema.ema_scan(x.cpu().numpy(), alpha.cpu().numpy())
    assert np.abs(y.numpy() - ref).max() < 1e-5
    check_device_status(x.device)
