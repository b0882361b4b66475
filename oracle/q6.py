"""CPU oracle: q6 KV codec -- TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Restates the engine-defined q6 format in numpy integer/float32 arithmetic
(the reference has no packed-KV path: kernels/dsqg_attention_v22.py:467).
Every step is done in IEEE float32 with round-to-nearest-even, so codes,
bytes and scales are bit-exact with the CUDA codec.
"""

from __future__ import annotations

import numpy as np


def pack(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """x[..., 64] float -> (codes uint8 [..., 48], scales float16 [...])."""
    x = np.asarray(x, dtype=np.float32)
    if x.shape[-1] != 64:
        raise ValueError("rows must have 64 values")
    amax = np.abs(x).max(axis=-1)
    scales = np.minimum(amax, np.float32(65504.0)).astype(np.float16)
    sf = scales.astype(np.float32)[..., None]
    with np.errstate(divide="ignore", invalid="ignore"):
        inv = np.float32(31.0) / sf                # one float32 division per row (RNE)
        q = np.rint(x * inv)                       # float32 multiply (RNE), round half to even
    q = np.where(sf > 0, q, np.float32(0.0))
    q = np.clip(q, -31, 31).astype(np.int32)
    u = (q & 63).astype(np.uint32).reshape(*x.shape[:-1], 16, 4)
    w = u[..., 0] | (u[..., 1] << 6) | (u[..., 2] << 12) | (u[..., 3] << 18)
    b = np.stack([w & 255, (w >> 8) & 255, (w >> 16) & 255], axis=-1).astype(np.uint8)
    return b.reshape(*x.shape[:-1], 48), scales


def codes(packed: np.ndarray) -> np.ndarray:
    """uint8 [..., 48] -> signed codes int32 [..., 64]."""
    b = np.asarray(packed, dtype=np.uint32).reshape(*packed.shape[:-1], 16, 3)
    w = b[..., 0] | (b[..., 1] << 8) | (b[..., 2] << 16)
    u = np.stack([(w >> (6 * i)) & 63 for i in range(4)], axis=-1).astype(np.int32)
    c = np.where(u >= 32, u - 64, u)
    return c.reshape(*packed.shape[:-1], 64)


def unpack(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """Dequantise to float32: float(c) * (float(s) / 31)."""
    step = (np.asarray(scales, dtype=np.float16).astype(np.float32) / np.float32(31.0))[..., None]
    return codes(packed).astype(np.float32) * step
