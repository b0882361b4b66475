import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def _device_status_stays_clear(request):
    """After every GPU test: no kernel hit its bounded-wait limit (the device status
    word is read and cleared; a timeout fails the test at teardown)."""
    yield
    if "gpu" not in request.keywords:
        return
    import torch

    if not torch.cuda.is_available():
        return
    from dwarf_v2_b200 import _lib

    _lib.check_device_status()
