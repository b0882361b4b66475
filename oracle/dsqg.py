"""CPU oracle: DSQG lattice attention -- TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Restates the reference DSQG forward in float64 numpy:

* semantics of ``_eager_dsqg_attention`` (kernels/dsqg_attention_v22.py:2602-2688):
  per query n and offset j, src = n - off[j], valid when src >= 0; score =
  (q . (k_src + E_j)) / sqrt(D) + pos_bias[j, h]; softmax over valid offsets;
  values of the large band rotated on four MOVT planes
  (``_rotate_sparse_value_eager`` :2560-2599);
* with the production kernel's precision choices (``_fwd_v22_online``
  :698-860): E_j rounded to bf16 before use (:760-763) and rotated values
  kept unrounded; rows before ``query_start`` are zero (:2267-2269).

Also the module-side probe projections (DSQGAttentionV19.forward :3231-3254)
and the parameter-derived tables (:2981-2995, 3256).
"""

from __future__ import annotations

import math

import numpy as np

R_PLANES = 4


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float values to the nearest bf16 (ties to even), returned as float64."""
    f = np.asarray(x, dtype=np.float32)
    bits = f.view(np.uint32).astype(np.uint64)
    rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
    return rounded.astype(np.uint32).view(np.float32).astype(np.float64)


def plane_channels(head_dim: int, plane_shift: int) -> list[tuple[int, int]]:
    stride = max(2, head_dim // R_PLANES)
    return [(r * stride + plane_shift, r * stride + plane_shift + 1) for r in range(R_PLANES)]


def dsqg_forward(q, k, v, pos_bias, scale_embed, phase_base, phase_gain, y_pre, z_pre, offsets,
                 j_small: int, plane_shift: int = 0, query_start: int = 0, round_scale_embed: bool = True):
    """All arrays float64-convertible; q [B,H,N,D], k/v [B,Hkv,N,D]. Returns (out [B,H,N,D], lse [B,H,N])."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    B, H, N, D = q.shape
    Hkv = k.shape[1]
    group = H // Hkv
    k = np.repeat(k, group, axis=1)
    v = np.repeat(v, group, axis=1)
    z = np.repeat(np.asarray(z_pre, np.float64), group, axis=1)
    y = np.asarray(y_pre, np.float64)
    se = bf16_round(scale_embed) if round_scale_embed else np.asarray(scale_embed, np.float64)
    pb = np.asarray(pos_bias, np.float64)
    pbase = np.asarray(phase_base, np.float64)
    pgain = np.asarray(phase_gain, np.float64)
    offsets = [int(o) for o in offsets]
    J = len(offsets)
    n = np.arange(N)
    scores = np.full((B, H, N, J), -np.inf)
    values = np.zeros((B, H, N, J, D))
    pairs = plane_channels(D, plane_shift)
    for j, delta in enumerate(offsets):
        src = n - delta
        valid = (src >= 0) & (n >= query_start)
        s = np.clip(src, 0, N - 1)
        ks, vs = k[:, :, s], v[:, :, s].copy()
        sc = (q * (ks + se[j])).sum(-1) / math.sqrt(D) + pb[j][None, :, None]
        scores[:, :, :, j] = np.where(valid[None, None], sc, -np.inf)
        if j >= j_small:
            jl = j - j_small
            zs = z[:, :, s]
            for r, (a, b) in enumerate(pairs):
                theta = pbase[jl, :, r][None, :, None] + pgain[jl, :, r][None, :, None] * y[..., r] * zs[..., r]
                c, sn = np.cos(theta), np.sin(theta)
                va, vb = vs[..., a].copy(), vs[..., b].copy()
                vs[..., a] = c * va - sn * vb
                vs[..., b] = sn * va + c * vb
        values[:, :, :, j] = vs
    m = scores.max(-1, keepdims=True)
    any_valid = np.isfinite(m)
    w = np.where(np.isfinite(scores), np.exp(scores - np.where(any_valid, m, 0.0)), 0.0)
    l = w.sum(-1, keepdims=True)
    out = np.where(l > 0, (w[..., None] * values).sum(-2) / np.where(l > 0, l, 1.0), 0.0)
    lse = np.where(l[..., 0] > 0, m[..., 0] + np.log(np.where(l[..., 0] > 0, l[..., 0], 1.0)), -np.inf)
    return out, lse


def probe_projection(x, probes) -> np.ndarray:
    """(x . p_r) / sqrt(|x|^2 + 1e-6 D) with L2-normalised probes (reference :3231-3254)."""
    x = np.asarray(x, np.float64)
    p = np.asarray(probes, np.float64)
    p = p / np.maximum(np.linalg.norm(p, axis=-1, keepdims=True), 1e-12)
    inv = 1.0 / np.sqrt((x * x).sum(-1, keepdims=True) + 1e-6 * x.shape[-1])
    return np.einsum("bhnd,rd->bhnr", x, p) * inv


def derived_tables(offsets, pos_bias_log_slope, pos_bias_residual, pos_bias_scale, scale_embed,
                   phase_base, phase_gain, phase_gate):
    """pos_bias, centred scale embedding, gated phase tables (reference :2981-2995, 3256)."""
    log_distance = np.log1p(np.asarray(offsets, np.float64))[:, None]
    slope = np.logaddexp(0.0, np.asarray(pos_bias_log_slope, np.float64))[None, :]
    pb = (-log_distance * slope + np.asarray(pos_bias_residual, np.float64)) * float(pos_bias_scale)
    se = np.asarray(scale_embed, np.float64)
    se = se - se.mean(0, keepdims=True)
    gate = 1.0 / (1.0 + np.exp(-np.asarray(phase_gate, np.float64)))[:, None, None]
    return pb, se, np.asarray(phase_base, np.float64) * gate, np.asarray(phase_gain, np.float64) * gate


def dsqg_forward_torch(q, k, v, pos_bias, scale_embed, phase_base, phase_gain, y_pre, z_pre, offsets,
                       j_small: int, plane_shift: int = 0, query_start: int = 0, round_scale_embed: bool = True):
    """``dsqg_forward`` restated on CPU torch tensors (any float dtype; use float64)
    so autograd can differentiate it: the oracle of the backward pass, whose
    gradients are those of ``_eager_dsqg_attention`` (dsqg_attention_v22.py:2602-2688)
    and of the reference backward kernels (:1263-2196, 2354-2552)."""
    import torch

    B, H, N, D = q.shape
    group = H // k.shape[1]
    kx, vx, zx = (t.repeat_interleave(group, dim=1) for t in (k, v, z_pre))
    se = scale_embed
    if round_scale_embed:
        se = se + (torch.from_numpy(bf16_round(scale_embed.detach().numpy())).to(se.dtype) - se).detach()
    n = torch.arange(N)
    pairs = plane_channels(D, plane_shift)
    scores, values = [], []
    for j, delta in enumerate(int(o) for o in offsets):
        src = n - delta
        valid = (src >= 0) & (n >= query_start)
        s = src.clamp(0, N - 1)
        ks, vs = kx[:, :, s], vx[:, :, s]
        sc = (q * (ks + se[j])).sum(-1) / math.sqrt(D) + pos_bias[j][None, :, None]
        scores.append(torch.where(valid[None, None], sc, torch.full_like(sc, -math.inf)))
        if j >= j_small:
            jl = j - j_small
            zs = zx[:, :, s]
            cols = list(vs.unbind(-1))
            for r, (a, b) in enumerate(pairs):
                theta = phase_base[jl, :, r][None, :, None] + phase_gain[jl, :, r][None, :, None] * y_pre[..., r] * zs[..., r]
                c, sn = torch.cos(theta), torch.sin(theta)
                va, vb = cols[a], cols[b]
                cols[a], cols[b] = c * va - sn * vb, sn * va + c * vb
            vs = torch.stack(cols, -1)
        values.append(vs)
    sc = torch.stack(scores, -1)
    any_valid = torch.isfinite(sc).any(-1, keepdim=True)
    p = torch.softmax(torch.where(any_valid, sc, torch.zeros_like(sc)), -1)
    p = torch.where(torch.isfinite(sc), p, torch.zeros_like(p))
    return (p.unsqueeze(-1) * torch.stack(values, -2)).sum(-2)


def dsqg_backward(inputs: dict, dout, offsets, j_small: int, plane_shift: int = 0, query_start: int = 0,
                  round_scale_embed: bool = True) -> dict:
    """Gradients (float64) of ``dsqg_forward_torch`` for dO = ``dout``; ``inputs``
    maps q, k, v, pos_bias, scale_embed, phase_base, phase_gain, y_pre, z_pre to
    tensors. Returns {'d_' + name: gradient}."""
    import torch

    names = ("q", "k", "v", "pos_bias", "scale_embed", "phase_base", "phase_gain", "y_pre", "z_pre")
    leaves = {n: torch.as_tensor(inputs[n]).double().clone().requires_grad_(True) for n in names}
    out = dsqg_forward_torch(*(leaves[n] for n in names), offsets, j_small, plane_shift, query_start,
                             round_scale_embed)
    grads = torch.autograd.grad(out, [leaves[n] for n in names], torch.as_tensor(dout).double(),
                                allow_unused=True)
    return {f"d_{n}": (g if g is not None else torch.zeros_like(leaves[n])) for n, g in zip(names, grads)}
