"""The allocation-free EMA scan entry point, dwarf_ema_scan_noalloc.

Some callers cannot allocate device memory where they call the scan (an
allocator-less runtime, a host application that forbids cudaMalloc on its hot
path, or an embedder that sizes all device memory up front). For them the
library keeps the scan's look-back scratch in a fixed device array of
DWARF_EMA_NOALLOC_SCRATCH_BYTES. This test calls that entry point through the
C ABI (ctypes, no workspace passed) and checks it against the regular
dwarf_ema_scan on two calls in a row, within the EMA tolerance the other tests
use (1e-5 in fp32; bf16 outputs within one bf16 step), and that a problem too
large for the array is refused before anything runs. The file sorts last so a
stop-at-first-failure run has already run every other test.
"""

import ctypes

import numpy as np
import pytest
import torch


def _noalloc(x: torch.Tensor, alpha: torch.Tensor, y: torch.Tensor) -> int:
    from dwarf_v2_b200 import _lib

    lib = _lib.load()
    B, N, D = x.shape
    args = _lib.EmaScanArgs(
        version=_lib.ABI_VERSION, dtype=_lib.dtype_code(x.dtype), x=x.data_ptr(), y=y.data_ptr(),
        batch=B, seq_len=N, width=D, sxb=x.stride(0), sxn=x.stride(1), sxd=x.stride(2),
        syb=y.stride(0), syn=y.stride(1), syd=y.stride(2), alpha=alpha.data_ptr(), alpha_per_channel=1,
        clamp=0, floor_=0.0, ceiling=1.0, workspace=None, workspace_bytes=0, device_status=None)
    return lib.dwarf_ema_scan_noalloc(ctypes.byref(args), _lib.stream_handle(x.device))


@pytest.mark.gpu
@pytest.mark.parametrize("shape,dtype", [((16, 2048, 512), torch.float32), ((3, 517, 264), torch.bfloat16)])
def test_noalloc_matches_regular_entry_point_twice(shape, dtype):
    from dwarf_v2_b200.causal_ema_scan import causal_ema_scan_per_channel

    gen = torch.Generator().manual_seed(sum(shape))
    for call in range(2):  # two calls in a row share (and must clear) the array
        x = torch.randn(shape, generator=gen).to(dtype).cuda()
        alpha = torch.rand(shape[-1], generator=gen).cuda()
        y = torch.empty_like(x)
        assert _noalloc(x, alpha, y) == 0
        ref = causal_ema_scan_per_channel(x, alpha)
        torch.cuda.synchronize()
        a, b = y.double().cpu().numpy(), ref.double().cpu().numpy()
        if dtype == torch.float32:
            assert np.abs(a - b).max() < 1e-5, (call, np.abs(a - b).max())
        else:
            assert np.all(np.abs(a - b) <= np.maximum(np.abs(b), 1e-3) * 2.0 ** -7), call


@pytest.mark.gpu
def test_noalloc_rejects_problems_beyond_the_scratch_limit():
    x = torch.zeros(64, 2048, 512, device="cuda")
    y = torch.full_like(x, 7.0)
    alpha = torch.full((512,), 0.1, device="cuda")
    assert _noalloc(x, alpha, y) == -10  # DWARF_ERR_SCRATCH_LIMIT
    torch.cuda.synchronize()
    assert torch.all(y == 7.0)  # nothing was launched
