"""Loads the committed golden fixtures (tests/golden/*.npz) as torch tensors."""

from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name: str) -> dict[str, torch.Tensor]:
    data = np.load(GOLDEN / f"{name}.npz")
    out = {}
    for key in data.files:
        arr = data[key]
        if key.endswith("__bf16"):
            out[key[: -len("__bf16")]] = torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16)
        else:
            out[key] = torch.from_numpy(np.ascontiguousarray(arr))
    return out
