"""CPU oracle: causal EMA scan -- TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Restates ``_reference`` (kernels/causal_ema_scan.py:511-538): a serial scan
``state = alpha*x[t] + (1-alpha)*state`` from ``state = 0`` with the state in
the accumulator dtype (fp64 here), output cast back to the input dtype by the
caller. ``alpha`` may be one scalar (reference API; clamped to [floor,ceiling]
as at :518) or one value per channel (unclamped, the per-channel config).
"""

from __future__ import annotations

import numpy as np


def ema_scan(x: np.ndarray, alpha, *, clamp: tuple[float, float] | None = None) -> np.ndarray:
    """x: [B,N,D] array (any float dtype); alpha: scalar or [D]. Returns fp64 [B,N,D]."""
    xf = np.asarray(x, dtype=np.float64)
    a = np.asarray(alpha, dtype=np.float64)
    if clamp is not None:
        a = np.clip(a, clamp[0], clamp[1])
    a = np.broadcast_to(a.reshape(-1) if a.ndim else a, (xf.shape[2],)).astype(np.float64)
    decay = 1.0 - a
    state = np.zeros((xf.shape[0], xf.shape[2]), dtype=np.float64)
    out = np.empty_like(xf)
    for t in range(xf.shape[1]):
        state = a * xf[:, t] + decay * state
        out[:, t] = state
    return out


def ema_scan_decay_form(x: np.ndarray, decay_a: np.ndarray) -> np.ndarray:
    """``y_t = a*y_{t-1} + (1-a)*x_t`` per channel: the same scan with alpha = 1 - a."""
    return ema_scan(x, 1.0 - np.asarray(decay_a, dtype=np.float64))
