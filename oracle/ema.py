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


def ema_scan_backward(x: np.ndarray, y: np.ndarray, dy: np.ndarray, alpha, *, per_channel: bool = False):
    """Gradients of ``ema_scan`` (reference _bwd_local/_bwd_carry/_bwd_apply,
    kernels/causal_ema_scan.py:157-260; _CausalEMAFn.backward :315-364).

    ``alpha`` is the (already clamped) scalar or per-channel factor, ``y`` the
    forward output. Reverse-time state ``s[t] = dy[t] + (1-alpha) s[t+1]``,
    ``dx = alpha * s`` and ``d alpha = sum s[t] * (x[t] - y[t-1])`` (y[-1] = 0),
    summed over (b, t) per channel, and over channels too for a scalar alpha.
    Returns fp64 (dx [B,N,D], d_alpha [D] or scalar); the clamp's projected
    derivative (:355-363) is the caller's.
    """
    xf, yf, g = (np.asarray(a, dtype=np.float64) for a in (x, y, dy))
    a = np.asarray(alpha, dtype=np.float64).reshape(-1)
    a = np.broadcast_to(a, (xf.shape[2],))
    decay = 1.0 - a
    state = np.zeros((xf.shape[0], xf.shape[2]), dtype=np.float64)
    dx = np.empty_like(xf)
    da = np.zeros(xf.shape[2], dtype=np.float64)
    for t in range(xf.shape[1] - 1, -1, -1):
        state = g[:, t] + decay * state
        dx[:, t] = a * state
        prev = yf[:, t - 1] if t > 0 else 0.0
        da += (state * (xf[:, t] - prev)).sum(axis=0)
    return dx, (da if per_channel else da.sum())
