"""Generates the golden fixtures in tests/golden/ by running the REFERENCE code.

Run in a container that has the reference checkout (path in DWARF_REFERENCE_DIR,
default ``/root/reference``); the fixtures it writes are committed and the
tests read only those files, so nothing at test time needs the reference.

    python tests/golden/make_golden.py [ema|dsqg|hisa|model|all]

Each fixture is an ``.npz`` holding the seeded inputs and the reference output
of one call, named for the reference function it exercises. bf16 tensors are
stored as their uint16 bit patterns (key suffix ``__bf16``).
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REFERENCE = Path(os.environ.get("DWARF_REFERENCE_DIR", "/root/reference"))


def _import_reference():
    for sub in ("kernels", "train"):
        path = str(REFERENCE / sub)
        if path not in sys.path:
            sys.path.insert(0, path)


def to_np(tensor: torch.Tensor) -> tuple[str, np.ndarray]:
    tensor = tensor.detach().cpu()
    if tensor.dtype == torch.bfloat16:
        return "__bf16", tensor.view(torch.int16).numpy().view(np.uint16)
    return "", tensor.numpy()


def save(name: str, **arrays) -> None:
    out = {}
    for key, value in arrays.items():
        if isinstance(value, torch.Tensor):
            suffix, arr = to_np(value)
            out[key + suffix] = arr
        else:
            out[key] = np.asarray(value)
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print("wrote", name, {k: v.shape for k, v in out.items()})


def make_ema() -> None:
    _import_reference()
    import causal_ema_scan as ref

    # The reference's own __main__ case (causal_ema_scan.py:570-581), forward only.
    torch.manual_seed(1)
    x = torch.randn(2, 9, 7, dtype=torch.float64)
    raw = torch.tensor(ref.inverse_bounded_ema_factor(0.05), dtype=torch.float64)
    alpha = ref.bounded_ema_factor(raw)
    y = ref.causal_ema_scan(x, alpha)
    save("ema_reference_main_f64", x=x, alpha=alpha.reshape(1), y=y)

    # fp32, alpha above the ceiling (clamped to 0.5), ragged sizes.
    g = torch.Generator().manual_seed(11)
    x = torch.randn(3, 200, 96, generator=g, dtype=torch.float32)
    alpha = torch.tensor([0.7], dtype=torch.float32)
    y = ref.causal_ema_scan(x, alpha)
    save("ema_scalar_clamped_f32", x=x, alpha=alpha, y=y)

    # bf16 input as the model feeds it (train_dwarf.py:261), alpha = 1/16.
    g = torch.Generator().manual_seed(12)
    x = torch.randn(2, 130, 512, generator=g).to(torch.bfloat16)
    alpha = torch.tensor([1.0 / 16.0], dtype=torch.float32)
    y = ref.causal_ema_scan(x, alpha)
    save("ema_scalar_bf16", x=x, alpha=alpha, y=y)

    # Per-channel decay (y_t = a*y_{t-1} + (1-a)*x_t, a = sigmoid(N(0,1))): the
    # reference _reference broadcasts a [D] alpha, so alpha = 1-a with bounds
    # that never bind reproduces it.
    g = torch.Generator().manual_seed(13)
    x = torch.randn(2, 300, 64, generator=g, dtype=torch.float32)
    decay = torch.sigmoid(torch.randn(64, generator=g))
    y = ref._reference(x, 1.0 - decay, 1e-12, 1.0 - 1e-12)
    save("ema_per_channel_f32", x=x, decay=decay, y=y)


def main(argv: list[str]) -> None:
    which = argv[1] if len(argv) > 1 else "all"
    makers = {"ema": make_ema}
    for name, maker in makers.items():
        if which in ("all", name):
            maker()


if __name__ == "__main__":
    main(sys.argv)
