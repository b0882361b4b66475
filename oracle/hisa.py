"""CPU oracle: V16/V18 HISA L3 mixer -- TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Restates, in numpy, the reference functions of
kernels/hierarchical_sparse_attn_v18_hisa.py used by the production forward
(eval mode, ``enumerate_all`` token selection, split lanes):

* ``chunk_representatives``  <- ``_completed_chunk_representatives`` (:171-219)
* ``select_chunks``          <- forward :2614-2624, ``_eligibility`` (:222-237),
  ``_build_causal_tile_metadata`` (:290-397): top-k over eligible completed
  chunks, -1 where the value is not finite; ties go to the LOWER chunk index
  (a stable sort), which the reference's ``torch.topk`` leaves unspecified.
* ``route_scores``           <- ``_selected_route_scores`` (:418-468)
* ``attention``              <- ``_eager_local_lane`` (:688-741) +
  ``_eager_global_lane`` (:744-805) + ``_merge_attention_lanes`` (:808-835),
  written as the one softmax over the union of both lanes that the exact LSE
  merge equals.

The router functions run in float32 with a fixed left-to-right summation
order (the order the CUDA kernels use), so chunk indices compare bit for bit;
``attention`` runs in float64.
"""

from __future__ import annotations

import math

import numpy as np

from .dsqg import bf16_round


def _f32(x):
    return np.asarray(x, dtype=np.float32)


def seq_sum(terms: np.ndarray, axis: int) -> np.ndarray:
    """float32 sum along `axis`, added strictly left to right."""
    terms = np.moveaxis(_f32(terms), axis, 0)
    acc = np.zeros(terms.shape[1:], np.float32)
    for i in range(terms.shape[0]):
        acc = acc + terms[i]
    return acc


def seq_dot(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """float32 dot over the last axis: products rounded, summed left to right."""
    return seq_sum(_f32(a) * _f32(b), axis=-1)


def l2_normalize_bf16(x: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """F.normalize(x.float(), eps).to(bf16) with a sequential float32 norm."""
    x = _f32(x)
    norm = np.sqrt(seq_sum(x * x, axis=-1))[..., None]
    return bf16_round(x / np.maximum(norm, np.float32(eps)).astype(np.float32))


def chunk_representatives(key, valid_lengths, chunk_size: int = 64, blend_alpha: float = 0.5) -> np.ndarray:
    """key [B,H,T,D] (bf16-valued) -> bf16-valued reps [B,H,C,D] (mean/max-L2 blend, L2-normalised)."""
    key = _f32(key)
    B, H, T, D = key.shape
    C = max(1, math.ceil(T / chunk_size))
    pad = C * chunk_size - T
    if pad:
        key = np.concatenate([key, np.zeros((B, H, pad, D), np.float32)], axis=2)
    chunks = key.reshape(B, H, C, chunk_size, D)
    ids = np.arange(C * chunk_size).reshape(C, chunk_size)
    lengths = np.asarray(valid_lengths).reshape(B, 1, 1)
    token_valid = (ids[None] < lengths)[:, None]                    # [B,1,C,S]
    valid_f = token_valid.astype(np.float32)[..., None]
    count = np.maximum(valid_f.sum(3), 1.0).astype(np.float32)
    mean = seq_sum(chunks * valid_f, axis=3) / count
    energy = seq_sum(chunks * chunks, axis=-1)                      # [B,H,C,S]
    energy = np.where(token_valid, energy, -np.inf)
    best = np.argmax(energy, axis=-1)                               # first maximum
    max_vec = np.take_along_axis(chunks, best[..., None, None], axis=3)[:, :, :, 0]
    a = np.float32(blend_alpha)
    rep = (np.float32(1.0) - a) * mean + a * max_vec
    norm = np.sqrt(seq_sum(rep * rep, axis=-1))[..., None]
    rep = rep / np.maximum(norm, np.float32(1e-6))
    chunk_valid = (np.arange(C) * chunk_size)[None] < np.asarray(valid_lengths).reshape(B, 1)
    rep = np.where(chunk_valid[:, None, :, None], rep, 0.0)
    return bf16_round(rep)


def select_chunks(query, reps, valid_lengths, *, chunk_size: int = 64, selector_tile: int = 16,
                  top_k: int = 4, temperature: float = 1.0):
    """Top-k eligible completed chunks per selector tile.

    Returns (top_idx int32 [B,H,tiles,K], logits float32 [B,H,tiles,C] masked to -inf).
    """
    q = _f32(query)
    B, H, T, D = q.shape
    C = reps.shape[2]
    tiles = math.ceil(T / selector_tile)
    starts = np.arange(tiles) * selector_tile
    anchor = l2_normalize_bf16(q[:, :, np.minimum(starts, T - 1)])
    logits = seq_dot(anchor[:, :, :, None, :], _f32(reps)[:, :, None, :, :])
    logits = logits / np.float32(temperature)
    lengths = np.asarray(valid_lengths).reshape(B, 1)
    chunk_start = np.arange(C) * chunk_size
    completed = (chunk_start + chunk_size)[None, :] <= starts[:, None]
    eligible = completed[None] & (chunk_start[None, None, :] < lengths[:, :, None]) & (
        starts[None, :, None] < lengths[:, :, None])
    masked = np.where(eligible[:, None], logits, -np.inf).astype(np.float32)
    k = min(top_k, C)
    order = np.argsort(-masked, axis=-1, kind="stable")[..., :k]
    values = np.take_along_axis(masked, order, axis=-1)
    top = np.where(np.isfinite(values), order, -1).astype(np.int32)
    return top, masked


def route_scores(query, reps, top_idx, route_scale, *, selector_tile: int = 16) -> np.ndarray:
    """[B,H,T,K] bf16-valued: (q^_n . rep_c - mean over valid slots) * scale[h], 0 for invalid slots."""
    q = _f32(query)
    B, H, T, D = q.shape
    qn = l2_normalize_bf16(q)
    tile = np.arange(T) // selector_tile
    idx = top_idx[:, :, tile]
    safe = np.maximum(idx, 0)
    bi = np.arange(B)[:, None, None, None]
    hi = np.arange(H)[None, :, None, None]
    sel = _f32(reps)[bi, hi, safe]
    s = seq_dot(qn[:, :, :, None, :], sel)
    valid = idx >= 0
    count = np.maximum(valid.sum(-1, keepdims=True), 1).astype(np.float32)
    mean = seq_sum(np.where(valid, s, np.float32(0.0)), axis=-1)[..., None] / count
    centered = np.where(valid, s - mean, np.float32(0.0))
    scaled = centered * _f32(route_scale).reshape(1, H, 1, 1)
    return bf16_round(scaled)


def attention(query, local_key, local_value, global_key, global_value, route, top_idx, valid_lengths, *,
              chunk_size: int = 64, selector_tile: int = 16, local_window: int = 64, heads=None) -> np.ndarray:
    """Joint softmax over the strict local window and the routed chunks; float64.

    ``heads`` optionally restricts the computation to a list of (b, h) pairs
    (other rows are left zero), which keeps full-length checks fast.
    """
    q = np.asarray(query, np.float64)
    B, H, T, D = q.shape
    scale = 1.0 / math.sqrt(D)
    lk, lv = np.asarray(local_key, np.float64), np.asarray(local_value, np.float64)
    gk, gv = np.asarray(global_key, np.float64), np.asarray(global_value, np.float64)
    route = np.asarray(route, np.float64)
    out = np.zeros_like(q)
    lengths = np.asarray(valid_lengths).reshape(B)
    K = top_idx.shape[-1]
    pairs = heads if heads is not None else [(b, h) for b in range(B) for h in range(H)]
    for b, h in pairs:
        vlen = int(min(lengths[b], T))
        for n in range(vlen):
            t = n // selector_tile
            loc = np.arange(max(0, n - local_window), n)
            ks, vs, bias = [lk[b, h, loc]], [lv[b, h, loc]], [np.zeros(loc.size)]
            for k in range(K):
                c = int(top_idx[b, h, t, k])
                if c < 0:
                    continue
                ids = np.arange(c * chunk_size, (c + 1) * chunk_size)
                ids = ids[(ids < n - local_window) & (ids < vlen)]
                ks.append(gk[b, h, ids])
                vs.append(gv[b, h, ids])
                bias.append(np.full(ids.size, route[b, h, n, k]))
            kk = np.concatenate(ks)
            if kk.shape[0] == 0:
                continue
            s = kk @ q[b, h, n] * scale + np.concatenate(bias)
            w = np.exp(s - s.max())
            out[b, h, n] = (w[:, None] * np.concatenate(vs)).sum(0) / w.sum()
    return out


def attention_torch(query, local_key, local_value, global_key, global_value, route, top_idx, valid_lengths, *,
                    chunk_size: int = 64, selector_tile: int = 16, local_window: int = 64):
    """``attention`` restated on CPU torch tensors, one selector tile at a time
    (its 16 queries against the tile's local window and routed chunks, masked),
    so autograd gives the gradients of the reference's lanes + merge
    (hierarchical_sparse_attn_v18_hisa.py:688-835; backward kernels :1103-1246).
    Differentiable in query, the four K/V tensors and route."""
    import torch

    B, H, T, D = query.shape
    scale = 1.0 / math.sqrt(D)
    lengths = torch.as_tensor(valid_lengths).reshape(B, 1, 1, 1).long()
    top = torch.as_tensor(top_idx).long()
    K = top.shape[-1]
    outs = []
    for t in range(-(-T // selector_tile)):
        n0, n1 = t * selector_tile, min((t + 1) * selector_tile, T)
        n = torch.arange(n0, n1)
        q = query[:, :, n0:n1]
        qv = n.reshape(1, 1, -1, 1) < lengths
        lids = torch.arange(n0 - local_window, n1 - 1)
        lmask = ((lids >= 0) & (lids[None] < n[:, None]) & (lids[None] >= n[:, None] - local_window))
        lmask = lmask.reshape(1, 1, n.numel(), -1) & (lids.reshape(1, 1, 1, -1) < lengths) & qv
        safe = lids.clamp(0, T - 1)
        s_loc = torch.einsum("bhqd,bhkd->bhqk", q, local_key[:, :, safe]) * scale
        c = top[:, :, t]                                              # [B,H,K]
        gids = c[..., None] * chunk_size + torch.arange(chunk_size)   # [B,H,K,C]
        gids = gids.reshape(B, H, K * chunk_size)
        gvalid = (c >= 0).repeat_interleave(chunk_size, dim=-1)
        gsafe = gids.clamp(0, T - 1)
        idx = gsafe[..., None].expand(-1, -1, -1, D)
        gk = torch.gather(global_key, 2, idx)
        gv = torch.gather(global_value, 2, idx)
        prior = route[:, :, n0:n1].repeat_interleave(chunk_size, dim=-1)
        s_glb = torch.einsum("bhqd,bhkd->bhqk", q, gk) * scale + prior
        gmask = (gvalid[:, :, None] & (gids[:, :, None] < n.reshape(1, 1, -1, 1) - local_window)
                 & (gids[:, :, None] < lengths) & qv)
        s = torch.cat([s_loc.expand(B, H, -1, -1), s_glb], -1)
        mask = torch.cat([lmask.expand(B, H, -1, -1), gmask], -1)
        s = s.masked_fill(~mask, float("-inf"))
        any_valid = mask.any(-1, keepdim=True)
        p = torch.softmax(torch.where(any_valid, s, torch.zeros_like(s)), -1)
        p = torch.where(mask, p, torch.zeros_like(p))
        v = torch.cat([local_value[:, :, safe].expand(B, H, -1, -1), gv], 2)
        outs.append(torch.einsum("bhqk,bhkd->bhqd", p, v))
    return torch.cat(outs, 2)


def attention_backward(inputs: dict, dout, top_idx, valid_lengths, **kw) -> dict:
    """float64 gradients of ``attention_torch`` for dO = ``dout``; ``inputs`` maps
    query, local_key, local_value, global_key, global_value, route to tensors."""
    import torch

    names = ("query", "local_key", "local_value", "global_key", "global_value", "route")
    leaves = {n: torch.as_tensor(inputs[n]).double().clone().requires_grad_(True) for n in names}
    out = attention_torch(*(leaves[n] for n in names), top_idx, valid_lengths, **kw)
    grads = torch.autograd.grad(out, [leaves[n] for n in names], torch.as_tensor(dout).double())
    return {f"d_{n}": g for n, g in zip(names, grads)}
