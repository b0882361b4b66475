"""HISA L3 mixer on B200: drop-in for the reference ``kernels/hierarchical_sparse_attn_v18_hisa.py``.

Public surface kept from the reference (same names, arguments, validation and
state_dict layout): ``HierarchicalSparseAttentionV16HISACausal`` (aliases V17,
V18) with ``forward(x, kv_inject=None, *, valid_lengths=None,
return_metadata=False, return_auxiliary=False)`` and ``prepare_runtime``;
``HISAMetadata``; ``HISASelectionCapture``.

Device pipeline of one inference forward (eval mode, no gradients):
one tcgen05 GEMM for qkvg and the adapters' rank-16 down-projections (one
weight, rows padded to 256), the two rank-16 up-projections (tcgen05, K = 16)
-> ``dwarf_npci_rotate``
(adapter add + EMA/NPCI rotation of global K and V, one pass each) ->
``dwarf_hisa_reps`` (chunk representatives) -> ``dwarf_hisa_select`` (tile
anchor logits, strict-causal top-k) -> ``dwarf_hisa_route`` -> ``dwarf_hisa_attn``
(route prior, local window and routed chunks in one softmax, S and P.V on
tcgen05 with TMEM accumulators) -> W_o GEMM (tcgen05) -> ``dwarf_gate_mul``
(the model fuses this gate into its residual add + RMSNorm).

Supported configuration: head_dim 64, chunk 64, selector tile 16, local
window 64, top_k <= 4, hisa_top_m_tokens >= chunk (the reference's
``enumerate_all`` path), representative modes mean_max_blend / mean / max_l2.
Metadata requested with ``return_metadata=True`` is the reference's canonical
listing: the routed chunk indices and, per (tile, slot), the chunk's valid
tokens in descending order of the tile anchor's score (``token_idx`` /
``token_scores``, ``enumerate_all=False``), built on the device from the same
router inputs; the attention itself attends every valid token of a routed
chunk either way.

Training mode, or any forward whose inputs or parameters need gradients, takes
``_forward_autograd``: the projections, adapters, NPCI rotation, chunk
representatives, route prior, exploration slot and router auxiliary loss as
torch ops on the device, the chunk selection on ``dwarf_hisa_select`` and the
attention on ``dwarf_hisa_attn`` / ``dwarf_hisa_attn_bwd``. Routing
diagnostics (entropy, attention mass) are not computed.
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib, gemm
from .glue import gate_mul
from .npci import npci_rotate_autograd, npci_rotate_cuda

_HD = 64
_CHUNK = 64
_TILE = 16
_WINDOW = 64
_MAX_TOP_K = 4


def _next_pow2(value: int) -> int:
    return 1 if value <= 1 else 1 << (int(value) - 1).bit_length()


def _is_power_of_two(value: int) -> bool:
    return value > 0 and value & (value - 1) == 0


def _inverse_softplus(value: float) -> float:
    value = float(value)
    if not math.isfinite(value) or value <= 0:
        raise ValueError("softplus target must be finite and positive")
    return math.log(math.expm1(value))


@dataclass(frozen=True)
class HISAMetadata:
    top_chunk_idx: torch.Tensor          # int32 [B,H,T,K]
    token_idx: torch.Tensor              # empty or int32 [B,H,T,K,M]
    token_scores: torch.Tensor           # empty or fp32 [B,H,T,K,M]
    tile_starts: torch.Tensor            # int32 [T]
    valid_lengths: torch.Tensor          # int32 [B]
    chunk_size: int
    selector_tile_size: int
    enumerate_all: bool


@dataclass(frozen=True)
class HISASelectionCapture:
    anchor_logits: torch.Tensor
    metadata: HISAMetadata
    auxiliary_loss: torch.Tensor


def _as_valid_lengths(lengths, *, batch_size: int, seq_len: int, device) -> torch.Tensor:
    """int32 [B] valid lengths (reference :82-96), range-checked on the host."""
    if lengths is None:
        return torch.full((batch_size,), seq_len, dtype=torch.int32, device=device)
    result = lengths.to(device=device, dtype=torch.int32).reshape(-1)
    if result.numel() != batch_size:
        raise ValueError(f"valid_lengths must contain {batch_size} entries")
    if not bool(((result >= 0) & (result <= seq_len)).all()):
        raise ValueError(f"valid_lengths must be in [0,{seq_len}]")
    return result.contiguous()


def _strides3(t):
    return t.stride(0), t.stride(1), t.stride(2)


def chunk_representatives(global_key: torch.Tensor, lengths: torch.Tensor, *, blend_alpha: float,
                          out: torch.Tensor | None = None, pos: torch.Tensor | None = None) -> torch.Tensor:
    """``dwarf_hisa_reps``: bf16 [B,H,ceil(T/64),64] normalised chunk representatives.

    With ``pos`` (device int64 [1]) only the chunk holding that position is rebuilt
    in ``out`` (a decode step; the other chunks keep their values)."""
    B, H, T, D = global_key.shape
    C = max(1, -(-T // _CHUNK))
    reps = torch.empty(B, H, C, D, dtype=torch.bfloat16, device=global_key.device) if out is None else out
    if tuple(reps.shape) != (B, H, C, D) or reps.dtype != torch.bfloat16 or not reps.is_contiguous():
        raise ValueError(f"reps must be a contiguous bf16 {(B, H, C, D)} tensor")
    args = _lib.HisaRepsArgs(version=_lib.ABI_VERSION, head_dim=D, chunk_size=_CHUNK, B=B, H=H, T=T,
                             key=global_key.data_ptr(), lengths=lengths.data_ptr(), blend_alpha=float(blend_alpha),
                             reps=reps.data_ptr(), pos=None if pos is None else pos.data_ptr())
    args.skb, args.skh, args.skn = _strides3(global_key)
    _lib.call("dwarf_hisa_reps", args, global_key.device)
    return reps


def select_chunks(query: torch.Tensor, reps: torch.Tensor, lengths: torch.Tensor, *, top_k: int,
                  temperature: float, want_logits: bool = False, tile_begin: int = 0, tile_count: int = 0,
                  pos: torch.Tensor | None = None):
    """``dwarf_hisa_select``: (top_chunk_idx int32 [B,H,tiles,K], optional masked logits).

    ``tile_begin``/``tile_count`` restrict the launch to selector tiles
    [tile_begin, tile_begin + tile_count) (count 0: every tile); other entries stay unset.
    ``pos`` (device int64 [1]) starts the window at tile pos // 16 at run time instead.
    """
    B, H, T, D = query.shape
    C = reps.shape[2]
    tiles = -(-T // _TILE)
    k_slots = min(int(top_k), C)
    top = torch.empty(B, H, tiles, k_slots, dtype=torch.int32, device=query.device)
    logits = torch.empty(B, H, tiles, C, dtype=torch.float32, device=query.device) if want_logits else None
    args = _lib.HisaSelectArgs(version=_lib.ABI_VERSION, head_dim=D, chunk_size=_CHUNK, selector_tile=_TILE,
                               top_k=int(top_k), B=B, H=H, T=T, query=query.data_ptr(), reps=reps.data_ptr(),
                               lengths=lengths.data_ptr(), temperature=float(temperature),
                               top_chunk_idx=top.data_ptr(), logits=None if logits is None else logits.data_ptr(),
                               tile_begin=int(tile_begin), tile_count=int(tile_count),
                               pos=None if pos is None else pos.data_ptr())
    args.sqb, args.sqh, args.sqn = _strides3(query)
    _lib.call("dwarf_hisa_select", args, query.device)
    return top, logits


def route_prior(query, reps, top, route_scale, *, tile_begin: int = 0, tile_count: int = 0,
                pos: torch.Tensor | None = None) -> torch.Tensor:
    """``dwarf_hisa_route``: bf16 route prior [B,H,T,4] of the selected chunks."""
    B, H, T, D = query.shape
    route = torch.empty(B, H, T, _MAX_TOP_K, dtype=torch.bfloat16, device=query.device)
    args = _lib.HisaRouteArgs(version=_lib.ABI_VERSION, head_dim=D, selector_tile=_TILE, k_slots=top.shape[-1],
                              B=B, H=H, T=T, C=reps.shape[2], query=query.data_ptr(), reps=reps.data_ptr(),
                              top_chunk_idx=top.data_ptr(), route_scale=route_scale.data_ptr(),
                              route=route.data_ptr(), tile_begin=int(tile_begin), tile_count=int(tile_count),
                              pos=None if pos is None else pos.data_ptr())
    args.sqb, args.sqh, args.sqn = _strides3(query)
    _lib.call("dwarf_hisa_route", args, query.device)
    return route


def tile_attention(query, local_key, local_value, global_key, global_value, reps, top, route_scale, lengths, *,
                   out: torch.Tensor | None = None, want_route: bool = False, tile_begin: int = 0,
                   tile_count: int = 0, pos: torch.Tensor | None = None):
    """``dwarf_hisa_route`` + ``dwarf_hisa_attn``: route prior, then local window + routed chunks.

    ``tile_begin``/``tile_count`` restrict both launches to the query rows of those selector
    tiles (count 0: every tile); ``out`` rows of other tiles are left untouched."""
    B, H, T, D = query.shape
    if out is None:
        out = torch.empty(B, H, T, D, dtype=torch.bfloat16, device=query.device)
    route = route_prior(query, reps, top, route_scale, tile_begin=tile_begin, tile_count=tile_count, pos=pos)
    args = _lib.HisaAttnArgs(version=_lib.ABI_VERSION, head_dim=D, chunk_size=_CHUNK, selector_tile=_TILE,
                             local_window=_WINDOW, k_slots=top.shape[-1], B=B, H=H, T=T,
                             query=query.data_ptr(), local_key=local_key.data_ptr(),
                             local_value=local_value.data_ptr(), global_key=global_key.data_ptr(),
                             global_value=global_value.data_ptr(), top_chunk_idx=top.data_ptr(),
                             route=route.data_ptr(), lengths=lengths.data_ptr(), out=out.data_ptr(),
                             tile_begin=int(tile_begin), tile_count=int(tile_count),
                             pos=None if pos is None else pos.data_ptr())
    args.sqb, args.sqh, args.sqn = _strides3(query)
    args.slkb, args.slkh, args.slkn = _strides3(local_key)
    args.slvb, args.slvh, args.slvn = _strides3(local_value)
    args.sgkb, args.sgkh, args.sgkn = _strides3(global_key)
    args.sgvb, args.sgvh, args.sgvn = _strides3(global_value)
    args.sob, args.soh, args.son = _strides3(out)
    _lib.call("dwarf_hisa_attn", args, query.device)
    return out, (route if want_route else None)


def _attn_launch(query, local_key, local_value, global_key, global_value, top, route, lengths, out, lse=None):
    """``dwarf_hisa_attn`` with a given bf16 route prior [B,H,T,4]; ``lse`` (fp32
    [B,H,T], optional) receives the row log-sum-exp (log2 units) the backward reads."""
    B, H, T, D = query.shape
    args = _lib.HisaAttnArgs(version=_lib.ABI_VERSION, head_dim=D, chunk_size=_CHUNK, selector_tile=_TILE,
                             local_window=_WINDOW, k_slots=top.shape[-1], B=B, H=H, T=T,
                             query=query.data_ptr(), local_key=local_key.data_ptr(),
                             local_value=local_value.data_ptr(), global_key=global_key.data_ptr(),
                             global_value=global_value.data_ptr(), top_chunk_idx=top.data_ptr(),
                             route=route.data_ptr(), lengths=lengths.data_ptr(), out=out.data_ptr(),
                             tile_begin=0, tile_count=0, pos=None, lse=None if lse is None else lse.data_ptr())
    args.sqb, args.sqh, args.sqn = _strides3(query)
    args.slkb, args.slkh, args.slkn = _strides3(local_key)
    args.slvb, args.slvh, args.slvn = _strides3(local_value)
    args.sgkb, args.sgkh, args.sgkn = _strides3(global_key)
    args.sgvb, args.sgvh, args.sgvn = _strides3(global_value)
    args.sob, args.soh, args.son = _strides3(out)
    _lib.call("dwarf_hisa_attn", args, query.device)


class _HisaAttnFn(torch.autograd.Function):
    """Differentiable fused tile attention: forward ``dwarf_hisa_attn``, backward
    ``dwarf_hisa_attn_bwd`` (the reference trains the same function as
    _GlobalHISATritonFn + autograd through the local lane and the LSE merge,
    hierarchical_sparse_attn_v18_hisa.py:1897-2027, 2424-2461, 808-835).
    Differentiable in query, the local and global K/V and the route prior;
    top_chunk_idx and lengths are routing decisions (no gradient)."""

    @staticmethod
    def forward(ctx, query, local_key, local_value, global_key, global_value, route, top, lengths):
        ins = [t.to(torch.bfloat16).contiguous() for t in (query, local_key, local_value, global_key, global_value,
                                                          route)]
        top = top.to(torch.int32).contiguous()
        B, H, T, D = ins[0].shape
        out = torch.empty(B, H, T, D, dtype=torch.bfloat16, device=query.device)
        lse = torch.empty(B, H, T, dtype=torch.float32, device=query.device)
        _attn_launch(*ins[:5], top, ins[5], lengths, out, lse)
        ctx.save_for_backward(*ins, top, lengths, out, lse)
        ctx.dtypes = tuple(t.dtype for t in (query, local_key, local_value, global_key, global_value, route))
        return out if query.dtype == torch.bfloat16 else out.to(query.dtype)

    @staticmethod
    def backward(ctx, dout):
        q, lk, lv, gk, gv, route, top, lengths, out, lse = ctx.saved_tensors
        B, H, T, D = q.shape
        dob = dout.to(torch.bfloat16).contiguous()
        f32 = dict(dtype=torch.float32, device=q.device)
        dq, dlk, dlv, dgk, dgv = (torch.empty(B, H, T, D, **f32) for _ in range(5))
        droute = torch.empty(B, H, T, route.shape[-1], **f32)
        delta = torch.empty(B, H, T, **f32)
        args = _lib.HisaAttnBwdArgs(version=_lib.ABI_VERSION, k_slots=top.shape[-1], B=B, H=H, T=T,
                                    query=q.data_ptr(), local_key=lk.data_ptr(), local_value=lv.data_ptr(),
                                    global_key=gk.data_ptr(), global_value=gv.data_ptr(),
                                    top_chunk_idx=top.data_ptr(), route=route.data_ptr(), lengths=lengths.data_ptr(),
                                    out=out.data_ptr(), dout=dob.data_ptr(), dq=dq.data_ptr(),
                                    d_local_key=dlk.data_ptr(), d_local_value=dlv.data_ptr(),
                                    d_global_key=dgk.data_ptr(), d_global_value=dgv.data_ptr(),
                                    d_route=droute.data_ptr(), lse=lse.data_ptr(), delta=delta.data_ptr())
        _lib.call("dwarf_hisa_attn_bwd", args, q.device)
        grads = (dq, dlk, dlv, dgk, dgv, droute)
        return (*(g.to(dt) for g, dt in zip(grads, ctx.dtypes)), None, None)


def hisa_tile_attention(query, local_key, local_value, global_key, global_value, route, top_chunk_idx,
                        valid_lengths=None):
    """Fused tile attention with a given route prior [B,H,T,4] (differentiable when
    its inputs require grad): one softmax over the strict local window (64) and the
    routed chunks of ``top_chunk_idx`` with ids < n - 64, route added per slot."""
    _lib.require_cuda(query, local_key, local_value, global_key, global_value, route)
    B, H, T, D = query.shape
    if D != _HD:
        raise ValueError(f"the B200 HISA kernels support head_dim 64, got {D}")
    if route.shape != (B, H, T, _MAX_TOP_K) or top_chunk_idx.shape[:3] != (B, H, -(-T // _TILE)):
        raise ValueError("route must be [B,H,T,4] and top_chunk_idx [B,H,ceil(T/16),K]")
    if top_chunk_idx.shape[-1] > _MAX_TOP_K:
        raise ValueError("at most 4 routed chunks per tile")
    lengths = _as_valid_lengths(valid_lengths, batch_size=B, seq_len=T, device=query.device)
    return _HisaAttnFn.apply(query, local_key, local_value, global_key, global_value, route, top_chunk_idx, lengths)


# ---------------------------------------------------------------------------
# Training-path router: differentiable device ops. The chunk selection itself
# comes from ``dwarf_hisa_select`` (integer decisions, no gradient); what the
# loss differentiates through -- the chunk representatives, the route prior of
# the selected chunks and the router's auxiliary loss -- is small next to the
# attention and is written here as torch ops on the device, as the reference
# writes it (its own training path is these ops under autograd).


def _chunk_view(key: torch.Tensor, lengths: torch.Tensor):
    """(chunks [B,H,C,64,D], token_valid [B,1,C,64], chunk_valid [B,C]) (reference :148-168)."""
    B, H, T, D = key.shape
    C = max(1, -(-T // _CHUNK))
    padded = F.pad(key, (0, 0, 0, C * _CHUNK - T)) if C * _CHUNK > T else key
    ids = torch.arange(C * _CHUNK, device=key.device, dtype=torch.int32).reshape(1, 1, C, _CHUNK)
    token_valid = ids < lengths.reshape(B, 1, 1, 1)
    starts = torch.arange(C, device=key.device, dtype=torch.int32) * _CHUNK
    chunk_valid = starts.reshape(1, C) < lengths.reshape(B, 1)
    return padded.reshape(B, H, C, _CHUNK, D), token_valid, chunk_valid


def representatives_autograd(global_key: torch.Tensor, lengths: torch.Tensor, blend_alpha: float) -> torch.Tensor:
    """Chunk representatives as differentiable ops: (1 - a) * mean + a * (row of largest
    squared norm, first on ties), L2-normalised (eps 1e-6), zero for chunks starting at
    or past the valid length, in the key's dtype (reference
    ``_completed_chunk_representatives``, hierarchical_sparse_attn_v18_hisa.py:171-219;
    a = 0 is its "mean" mode, a = 1 its "max_l2" mode)."""
    chunks, token_valid, chunk_valid = _chunk_view(global_key, lengths)
    values = chunks.float()
    weight = token_valid.unsqueeze(-1).to(values.dtype)
    mean = (values * weight).sum(3) / weight.sum(3).clamp_min(1.0)
    energy = values.detach().square().sum(-1).masked_fill(~token_valid, float("-inf"))
    best = energy.argmax(-1, keepdim=True)
    peak = torch.gather(values, 3, best.unsqueeze(-1).expand(-1, -1, -1, 1, values.shape[-1])).squeeze(3)
    rep = F.normalize((1.0 - blend_alpha) * mean + blend_alpha * peak, dim=-1, eps=1e-6)
    return rep.masked_fill(~chunk_valid[:, None, :, None], 0.0).to(global_key.dtype)


def _eligible(tiles: int, num_chunks: int, lengths: torch.Tensor) -> torch.Tensor:
    """bool [B, tiles, C]: chunk complete before the tile starts, chunk and tile inside the
    valid length (reference ``_eligibility``, :222-237)."""
    device = lengths.device
    tile_starts = torch.arange(tiles, device=device, dtype=torch.int32) * _TILE
    chunk_starts = torch.arange(num_chunks, device=device, dtype=torch.int32) * _CHUNK
    tile_valid = tile_starts.reshape(1, -1) < lengths.reshape(-1, 1)
    chunk_valid = chunk_starts.reshape(1, -1) < lengths.reshape(-1, 1)
    completed = (chunk_starts + _CHUNK).reshape(1, 1, -1) <= tile_starts.reshape(1, -1, 1)
    return completed & chunk_valid[:, None, :] & tile_valid[:, :, None]


def inject_exploration(top: torch.Tensor, eligible: torch.Tensor, probability: float) -> torch.Tensor:
    """With probability ``probability`` per (b, h, tile), the last slot of ``top`` is
    replaced by a uniformly drawn eligible chunk that is not selected yet (reference
    ``_inject_exploration_slot``, :240-287: the same draws, ``torch.rand`` over
    [B,H,tiles,C] then over [B,H,tiles], on the device)."""
    if probability <= 0.0 or top.shape[-1] == 0:
        return top
    B, H, tiles, slots = top.shape
    valid = top >= 0
    counts = torch.zeros(B, H, tiles, eligible.shape[-1], dtype=torch.int32, device=top.device)
    counts.scatter_add_(-1, top.clamp_min(0).long(), valid.to(torch.int32))
    candidate = eligible[:, None].expand(-1, H, -1, -1) & ~(counts > 0)
    random_scores = torch.rand(candidate.shape, device=top.device).masked_fill(~candidate, -1.0)
    best_value, best_choice = random_scores.max(-1)
    replace = (torch.rand(B, H, tiles, device=top.device) < probability) & (best_value >= 0.0)
    result = top.clone()
    result[..., slots - 1] = torch.where(replace, best_choice.to(result.dtype), result[..., slots - 1])
    return result.contiguous()


def selected_route_scores(query_normalized: torch.Tensor, reps: torch.Tensor, top: torch.Tensor,
                          route_scale: torch.Tensor) -> torch.Tensor:
    """Route prior [B,H,T,4] of the selected chunks as differentiable ops: per query and
    slot, q̂ . rep minus the mean over the tile's valid slots, times the head's scale; 0
    for invalid and padding slots; in the query's dtype (reference ``_selected_route_scores``,
    :418-468)."""
    B, H, T, D = query_normalized.shape
    tiles, K = top.shape[2], top.shape[3]
    padded = tiles * _TILE
    q = F.pad(query_normalized, (0, 0, 0, padded - T)) if padded > T else query_normalized
    q = q.reshape(B, H, tiles, _TILE, D)
    b_idx = torch.arange(B, device=top.device).reshape(B, 1, 1, 1)
    h_idx = torch.arange(H, device=top.device).reshape(1, H, 1, 1)
    selected = reps[b_idx, h_idx, top.clamp_min(0).long()]
    scores = torch.einsum("bhtsd,bhtkd->bhtsk", q.float(), selected.float())
    valid = (top >= 0)[..., None, :]
    count = valid.sum(-1, keepdim=True).clamp_min(1)
    mean = (scores * valid).sum(-1, keepdim=True) / count
    centred = torch.where(valid, scores - mean, torch.zeros_like(scores))
    scaled = centred * route_scale.reshape(1, H, 1, 1, 1).float()
    route = scaled.reshape(B, H, padded, K)[:, :, :T].to(query_normalized.dtype)
    return F.pad(route, (0, _MAX_TOP_K - K)) if K < _MAX_TOP_K else route


def router_auxiliary_loss(anchor_logits: torch.Tensor, anchor_query: torch.Tensor, global_key: torch.Tensor,
                          lengths: torch.Tensor, *, samples: int, temperature: float) -> torch.Tensor:
    """Cross entropy of the anchor routing against the token-level chunk evidence
    (logsumexp over each eligible chunk's q . k / 8) of up to ``samples`` selector tiles
    drawn without replacement (all of them when that covers every candidate tile)
    (reference ``_router_auxiliary_loss``, :471-531)."""
    if samples <= 0:
        return anchor_logits.sum() * 0.0
    B, H, tiles, C = anchor_logits.shape
    eligible_all = _eligible(tiles, C, lengths)
    first_useful = -(-_CHUNK // _TILE)
    candidates = max(0, tiles - first_useful)
    if candidates == 0:
        return anchor_logits.sum() * 0.0
    count = min(int(samples), candidates)
    useful = torch.arange(first_useful, tiles, device=anchor_logits.device, dtype=torch.long)
    tile_ids = useful if count == candidates else useful[torch.randperm(candidates, device=anchor_logits.device)[:count]]
    chunks, token_valid, _ = _chunk_view(global_key, lengths)
    query = anchor_query[:, :, tile_ids].float()
    token_scores = torch.einsum("bhsd,bhcmd->bhscm", query, chunks.float()) / math.sqrt(global_key.shape[-1])
    eligible = eligible_all[:, tile_ids]
    mask = token_valid[:, :, None] & eligible[:, None, :, :, None]
    evidence = torch.logsumexp(token_scores.masked_fill(~mask, -1e9), dim=-1)
    route = anchor_logits[:, :, tile_ids].float().masked_fill(~eligible[:, None], -1e9)
    target = torch.softmax((evidence / float(temperature)).detach(), dim=-1)
    per_row = -(target * torch.log_softmax(route, dim=-1)).sum(-1)
    valid_rows = eligible.any(-1)[:, None].expand(-1, H, -1)
    return (per_row * valid_rows).sum() / valid_rows.sum().clamp_min(1)


def hisa_attention(query, local_key, local_value, global_key, global_value, route_scale, valid_lengths=None, *,
                   top_k: int = 4, temperature: float = 1.0, blend_alpha: float = 0.5, want_route: bool = False):
    """Router + fused attention on head tensors [B,H,T,64] (bf16).

    Returns (output bf16 [B,H,T,64], top_chunk_idx, route bf16 [B,H,T,4] or None).
    """
    _lib.require_cuda(query, local_key, local_value, global_key, global_value)
    if torch.is_grad_enabled() and query.requires_grad:
        raise NotImplementedError("dwarf_v2_b200 is a forward (inference) engine; run under torch.no_grad()")
    B, H, T, D = query.shape
    if D != _HD:
        raise ValueError(f"the B200 HISA kernels support head_dim 64, got {D}")
    if -(-T // _CHUNK) > 128:
        raise ValueError("the B200 HISA router supports up to 128 chunks (T <= 8192)")
    lengths = _as_valid_lengths(valid_lengths, batch_size=B, seq_len=T, device=query.device)
    scale = route_scale.detach().reshape(-1).to(device=query.device, dtype=torch.float32).contiguous()
    reps = chunk_representatives(global_key, lengths, blend_alpha=blend_alpha)
    top, _ = select_chunks(query, reps, lengths, top_k=top_k, temperature=temperature)
    out, route = tile_attention(query, local_key, local_value, global_key, global_value, reps, top, scale, lengths,
                                want_route=want_route)
    return out, top, route


def _magnitude_aware_rotate(x, delta, theta_h, *, strength_tau: float = 0.25):
    """Norm-preserving tangent rotation (reference :99-125), one CUDA kernel."""
    return npci_rotate_cuda(x, delta, theta_h, strength_tau=strength_tau)


def _to_heads(t: torch.Tensor, batch: int, seq_len: int, heads: int, head_dim: int) -> torch.Tensor:
    return t.reshape(batch, seq_len, heads, head_dim).permute(0, 2, 1, 3)


class HierarchicalSparseAttentionV16HISACausal(nn.Module):
    """HISA V18 strict-causal L3 mixer with the reference's parameters (reference :2183-2787)."""

    def __init__(self, D: int, H: int, hd: int, num_chunks: int = 32, top_k_chunks: int = 4,
                 hisa_top_m_tokens: int = 64, *, chunk_size: int | None = None, local_window: int | None = None,
                 selector_tile_size: int | None = None, temperature: float = 1.0, route_prior_scale: float = 0.1,
                 backend: str | None = None, token_selection_mode: str | None = None,
                 representative_mode: str = "mean_max_blend", representative_blend_alpha: float = 0.5,
                 exploration_probability: float = 0.05, route_aux_weight: float = 0.01,
                 route_aux_samples: int = 4, route_aux_temperature: float = 1.0, global_adapter_rank: int = 16,
                 npci_theta_max: float = 0.25, max_seq_len: int | None = None, local_backend: str = "flex",
                 collect_routing_diagnostics: bool | None = None, diagnostic_max_queries: int | None = None) -> None:
        super().__init__()
        D, H, hd = int(D), int(H), int(hd)
        if D != H * hd:
            raise ValueError(f"D={D} must equal H*hd={H * hd}")
        if not _is_power_of_two(hd):
            raise ValueError("HISA head dimension must be a power of two")
        if top_k_chunks < 1 or hisa_top_m_tokens < 1:
            raise ValueError("top_k_chunks and hisa_top_m_tokens must be positive")
        if not math.isfinite(temperature) or temperature <= 0:
            raise ValueError("temperature must be finite and positive")
        if not math.isfinite(route_prior_scale) or route_prior_scale <= 0:
            raise ValueError("route_prior_scale must be finite and positive")
        if not 0.0 <= exploration_probability <= 1.0:
            raise ValueError("exploration_probability must be in [0,1]")
        if route_aux_weight < 0 or route_aux_samples < 0:
            raise ValueError("route auxiliary weight/samples must be non-negative")
        if not math.isfinite(route_aux_temperature) or route_aux_temperature <= 0:
            raise ValueError("route_aux_temperature must be finite and positive")
        if representative_mode not in {"max_l2", "mean", "mean_max_blend", "top2_blend"}:
            raise ValueError("unsupported representative_mode")
        if not 0.0 <= representative_blend_alpha <= 1.0:
            raise ValueError("representative_blend_alpha must be in [0,1]")
        if global_adapter_rank < 0:
            raise ValueError("global_adapter_rank must be non-negative")
        if not math.isfinite(npci_theta_max) or npci_theta_max <= 0:
            raise ValueError("npci_theta_max must be finite and positive")
        local_backend = str(local_backend).lower()
        if local_backend not in {"flex", "combined"}:
            raise ValueError("local_backend must be flex or combined")
        if max_seq_len is not None and int(max_seq_len) < 1:
            raise ValueError("max_seq_len must be positive when supplied")
        self.D, self.H, self.num_heads, self.hd = D, H, H, hd
        self.legacy_num_chunks = int(num_chunks)
        self.chunk_size = int(chunk_size if chunk_size is not None else os.getenv("DWARF_HISA_CHUNK_SIZE", "64"))
        self.local_window = int(local_window if local_window is not None
                                else os.getenv("DWARF_HISA_V16_LOCAL_WINDOW", "64"))
        self.selector_tile_size = int(selector_tile_size if selector_tile_size is not None
                                      else os.getenv("DWARF_HISA_V16_SELECTOR_TILE", "16"))
        if self.chunk_size < 1 or self.local_window < 1 or self.selector_tile_size < 1:
            raise ValueError("chunk_size, local_window, and selector_tile_size must be positive")
        self.top_k_chunks = int(top_k_chunks)
        self.hisa_top_m_tokens = int(hisa_top_m_tokens)
        self.temperature = float(temperature)
        self.backend = (backend or os.getenv("DWARF_HISA_V16_BACKEND", "auto")).lower()
        if self.backend not in {"auto", "eager", "triton"}:
            raise ValueError("backend must be auto, eager, or triton")
        self.token_selection_mode = (token_selection_mode
                                     or os.getenv("DWARF_HISA_V16_TOKEN_SELECTION", "auto")).lower()
        if self.token_selection_mode not in {"auto", "canonical"}:
            raise ValueError("token_selection_mode must be auto or canonical")
        self.representative_mode = representative_mode
        self.representative_blend_alpha = float(representative_blend_alpha)
        self.exploration_probability = float(exploration_probability)
        self.route_aux_weight = float(route_aux_weight)
        self.route_aux_samples = int(route_aux_samples)
        self.route_aux_temperature = float(route_aux_temperature)
        self.global_adapter_rank = int(global_adapter_rank)
        self.npci_theta_max = float(npci_theta_max)
        self.max_seq_len = None if max_seq_len is None else int(max_seq_len)
        self.local_backend = local_backend
        self.triton_block_q = int(os.getenv("DWARF_HISA_V16_BLOCK_Q", "16"))
        self.backward_impl = os.getenv("DWARF_HISA_V16_BWD", "atomic_masked").lower()
        if self.backward_impl not in {"atomic", "atomic_masked"}:
            raise ValueError("DWARF_HISA_V16_BWD must be atomic or atomic_masked")
        if collect_routing_diagnostics is None:
            collect_routing_diagnostics = os.getenv("DWARF_HISA_V16_ROUTING_DIAGNOSTICS", "0") == "1"
        self.collect_routing_diagnostics = bool(collect_routing_diagnostics)
        self.diagnostic_max_queries = int(diagnostic_max_queries or 8)
        if self.diagnostic_max_queries < 1:
            raise ValueError("diagnostic_max_queries must be positive")

        self.qkvg_proj = nn.Linear(D, 4 * D, bias=True)
        self.W_o = nn.Linear(D, D, bias=False)
        with torch.no_grad():
            self.qkvg_proj.bias.zero_()
        if self.global_adapter_rank:
            rank = self.global_adapter_rank
            self.global_k_down = nn.Linear(D, rank, bias=False)
            self.global_k_up = nn.Linear(rank, D, bias=False)
            self.global_v_down = nn.Linear(D, rank, bias=False)
            self.global_v_up = nn.Linear(rank, D, bias=False)
            nn.init.zeros_(self.global_k_up.weight)
            nn.init.zeros_(self.global_v_up.weight)
        else:
            self.global_k_down = self.global_k_up = self.global_v_down = self.global_v_up = None
        self.route_prior_raw = nn.Parameter(torch.full((H,), _inverse_softplus(route_prior_scale)))
        raw_theta = math.atanh(min(0.01 / max(self.npci_theta_max, 1e-6), 0.99))
        self.npci_theta_k = nn.Parameter(torch.full((H,), raw_theta))
        self.npci_theta_v = nn.Parameter(torch.full((H,), raw_theta))
        self._routing_entropy: torch.Tensor | float = float("nan")
        self._routing_diagnostics: dict[str, torch.Tensor] = {}
        self.hisa_evidence_capture: HISASelectionCapture | None = None
        self._routing_auxiliary_loss: torch.Tensor | None = None
        self._last_token_selection_path = ""

    @property
    def route_prior_scale(self) -> torch.Tensor:
        return F.softplus(self.route_prior_raw)

    def routing_auxiliary_loss(self, *, clear: bool = False) -> torch.Tensor | None:
        value = self._routing_auxiliary_loss
        if clear:
            self._routing_auxiliary_loss = None
        return value

    def semantic_config(self) -> dict[str, object]:
        return {
            "implementation": "hisa-v18-split-lse",
            "chunk_size": self.chunk_size,
            "top_k_chunks": self.top_k_chunks,
            "top_m_tokens": self.hisa_top_m_tokens,
            "local_window": self.local_window,
            "selector_tile_size": self.selector_tile_size,
            "temperature": self.temperature,
            "representative_mode": self.representative_mode,
            "representative_blend_alpha": self.representative_blend_alpha,
            "exploration_probability": self.exploration_probability,
            "route_aux_weight": self.route_aux_weight,
            "route_aux_samples": self.route_aux_samples,
            "route_aux_temperature": self.route_aux_temperature,
            "global_adapter_rank": self.global_adapter_rank,
            "npci_theta_max": self.npci_theta_max,
            "token_selection_mode": self.token_selection_mode,
            "selected_route_scoring": "tile_gather",
            "lane_merge": "exact_lse",
        }

    def execution_config(self) -> dict[str, object]:
        return {
            "backend": self.backend,
            "local_backend": "dwarf_hisa_attn",
            "attention_kernel": "mma.sync" if os.environ.get("DWARF_HISA_ATTN", "").startswith("m") else "tcgen05",
            "triton_block_q": self.triton_block_q,
            "backward_impl": self.backward_impl,
            # the two reference settings above are validated and echoed but select
            # nothing here: one forward and one backward kernel serve every value
            "ignored_settings": ("triton_block_q", "backward_impl"),
            "collect_routing_diagnostics": self.collect_routing_diagnostics,
            "flex_attention_available": False,
            "flex_lse_api": "none",
        }

    def _migrate_legacy_keys(self, state_dict, prefix: str) -> None:
        """Rewrites, in place, the reference's older checkpoint layouts (hierarchical_sparse_attn_v18_hisa.py:2469-2544).

        Separate ``W_q`` / ``W_k`` / ``W_v`` (+ biases, zero when absent) and the block's
        ``gate_proj`` (or ``global_gate``; zero when absent) -> one ``qkvg_proj``; parameters
        newer than the checkpoint (route prior, NPCI angles, global adapters) keep this
        module's current values.
        """
        w_key, b_key = prefix + "qkvg_proj.weight", prefix + "qkvg_proj.bias"
        if w_key not in state_dict:
            qw, kw, vw = (state_dict.get(prefix + f"{n}.weight") for n in ("W_q", "W_k", "W_v"))
            if qw is not None and kw is not None and vw is not None:
                parent = prefix[: -len("attn.")] if prefix.endswith("attn.") else prefix
                gw = state_dict.get(parent + "gate_proj.weight")
                if gw is None:
                    gw = state_dict.get(parent + "global_gate.weight")
                if gw is None:
                    gw = torch.zeros_like(qw)
                qb = state_dict.get(prefix + "W_q.bias", qw.new_zeros(qw.shape[0]))
                kb = state_dict.get(prefix + "W_k.bias", kw.new_zeros(kw.shape[0]))
                vb = state_dict.get(prefix + "W_v.bias", vw.new_zeros(vw.shape[0]))
                gb = state_dict.get(parent + "gate_proj.bias")
                if gb is None:
                    gb = state_dict.get(parent + "global_gate.bias")
                if gb is None:
                    gb = qw.new_zeros(qw.shape[0])
                state_dict[w_key] = torch.cat((qw, kw, vw, gw), dim=0)
                state_dict[b_key] = torch.cat((qb, kb, vb, gb), dim=0)
                for n in ("W_q.weight", "W_q.bias", "W_k.weight", "W_k.bias", "W_v.weight", "W_v.bias"):
                    state_dict.pop(prefix + n, None)
                for n in ("gate_proj.weight", "gate_proj.bias", "global_gate.weight", "global_gate.bias"):
                    state_dict.pop(parent + n, None)
        current = self.state_dict()
        for name in ("route_prior_raw", "npci_theta_k", "npci_theta_v", "global_k_down.weight",
                     "global_k_up.weight", "global_v_down.weight", "global_v_up.weight"):
            if name in current and prefix + name not in state_dict:
                state_dict[prefix + name] = current[name].detach().clone()

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                              error_msgs):
        self._migrate_legacy_keys(state_dict, prefix)
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                                      error_msgs)

    def prepare_runtime(self, device, seq_len: int | None = None) -> None:
        """Nothing to prebuild: the fused kernel needs no block mask."""
        return None

    def reset_global_adapters_(self) -> None:
        if self.global_adapter_rank:
            nn.init.zeros_(self.global_k_up.weight)
            nn.init.zeros_(self.global_v_up.weight)

    def _check_supported(self) -> None:
        if (self.hd, self.chunk_size, self.selector_tile_size, self.local_window) != (_HD, _CHUNK, _TILE, _WINDOW):
            raise NotImplementedError(
                "the B200 HISA kernels implement head_dim 64, chunk 64, selector tile 16, local window 64")
        if self.top_k_chunks > _MAX_TOP_K:
            raise NotImplementedError("the B200 HISA kernels route to at most 4 chunks per tile")
        if self.hisa_top_m_tokens < self.chunk_size:
            raise NotImplementedError("the B200 HISA kernels implement top_m_tokens >= chunk_size (enumerate_all)")
        if self.representative_mode == "top2_blend":
            raise NotImplementedError("representative_mode='top2_blend' is not implemented on B200")
        if self.backend == "eager":
            raise NotImplementedError("the B200 engine has no eager backend")

    @property
    def _blend_alpha(self) -> float:
        return {"mean": 0.0, "max_l2": 1.0}.get(self.representative_mode, self.representative_blend_alpha)

    def _projection_weights(self) -> tuple[torch.Tensor, torch.Tensor]:
        """One bf16 weight [qkvg_proj ; global_k_down ; global_v_down ; zero rows] (rows padded
        to a multiple of 256, the GEMM's wide tile) and its bias (zeros past qkvg), rebuilt only
        when a parameter changes: the input projection and the adapters' down-projections in
        one GEMM."""
        params = [self.qkvg_proj.weight, self.qkvg_proj.bias]
        if self.global_adapter_rank:
            params += [self.global_k_down.weight, self.global_v_down.weight]
        key = tuple((t.data_ptr(), t._version, t.dtype, t.device) for t in params)
        if getattr(self, "_proj_key", None) != key:
            with torch.no_grad():
                act = torch.bfloat16
                w = [self.qkvg_proj.weight.to(act)]
                b = [self.qkvg_proj.bias.to(act)]
                if self.global_adapter_rank:
                    w += [self.global_k_down.weight.to(act), self.global_v_down.weight.to(act)]
                    b.append(torch.zeros(2 * self.global_adapter_rank, dtype=act, device=b[0].device))
                rows = sum(t.shape[0] for t in w)
                pad = -rows % 256
                if pad:
                    w.append(torch.zeros(pad, w[0].shape[1], dtype=act, device=w[0].device))
                    b.append(torch.zeros(pad, dtype=act, device=b[0].device))
                self._proj = (torch.cat(w).contiguous(), torch.cat(b).contiguous())
            self._proj_key = key
        return self._proj

    def _project(self, xb: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor | None]:
        """(qkvg [B,T,4D], adapter down-projections [B,T,2r] or None) from one tcgen05 GEMM;
        both are column views of the GEMM's output."""
        weight, bias = self._projection_weights()
        out = gemm.linear(xb, weight, bias)
        D, r = self.D, self.global_adapter_rank
        return out[..., : 4 * D], (out[..., 4 * D: 4 * D + 2 * r] if r else None)

    def global_kv(self, x, local_key, local_value, kv_inject, down=None):
        """Global K/V = local + low-rank adapter, NPCI-rotated toward the packet deltas when given.
        ``down``: the adapters' down-projections of x when the caller already has them."""
        B, T, _ = x.shape
        act = torch.bfloat16
        addend_k = addend_v = None
        if self.global_adapter_rank:
            r = self.global_adapter_rank
            if down is None:  # callers outside the fused projection (N = 2r is below the GEMM's 128-column tile)
                down = F.linear(x, torch.cat((self.global_k_down.weight, self.global_v_down.weight)).to(act))
            addend_k = _to_heads(gemm.linear(down[..., :r], self.global_k_up.weight.to(act)), B, T, self.H, self.hd)
            addend_v = _to_heads(gemm.linear(down[..., r:], self.global_v_up.weight.to(act)), B, T, self.H, self.hd)
        kd = vd = None
        if kv_inject is not None:
            kd, vd = kv_inject
            if kd.shape != local_key.shape or vd.shape != local_value.shape:
                raise ValueError("kv_inject must contain [B,H,N,HD] tensors")
        if addend_k is None and kd is None:
            return local_key, local_value
        theta_k = self.npci_theta_max * torch.tanh(self.npci_theta_k.detach().float())
        theta_v = self.npci_theta_max * torch.tanh(self.npci_theta_v.detach().float())
        gk = npci_rotate_cuda(local_key, kd, theta_k, addend=addend_k)
        gv = npci_rotate_cuda(local_value, vd, theta_v, addend=addend_v)
        return gk, gv

    def forward_parts(self, x: torch.Tensor, kv_inject, lengths: torch.Tensor, *, router_inputs: list | None = None):
        """(W_o(attended), content-gate logits, top_chunk_idx): the forward up to the output gate.

        The model fuses ``* sigmoid(gate)`` into its residual-add + RMSNorm kernel.
        ``router_inputs``: a list that receives (query, global_key) for the metadata listing.
        """
        B, T, _ = x.shape
        act = torch.bfloat16
        xb = x if x.dtype == act else x.to(act)
        qkvg, down = self._project(xb)
        q, k, v, gate = qkvg.split(self.D, dim=-1)
        query = _to_heads(q, B, T, self.H, self.hd)
        local_key = _to_heads(k, B, T, self.H, self.hd)
        local_value = _to_heads(v, B, T, self.H, self.hd)
        global_key, global_value = self.global_kv(xb, local_key, local_value, kv_inject, down)
        attended = torch.empty(B, T, self.D, dtype=act, device=x.device)
        reps = chunk_representatives(global_key, lengths, blend_alpha=self._blend_alpha)
        top, _ = select_chunks(query, reps, lengths, top_k=self.top_k_chunks, temperature=self.temperature)
        scale = self.route_prior_scale.detach().float().contiguous()
        tile_attention(query, local_key, local_value, global_key, global_value, reps, top, scale, lengths,
                       out=_to_heads(attended, B, T, self.H, self.hd))
        self._last_token_selection_path = "enumerate_all"
        if router_inputs is not None:
            router_inputs.extend((query, global_key))
        return gemm.linear(attended, self.W_o.weight.to(act)), gate, top

    def forward_parts_cached(self, x: torch.Tensor, kv_inject, cache, row: int):
        """``forward_parts`` for positions [row, row + T) of ``x`` [B,T,D] over a cache.

        ``cache`` = (query, local_key, local_value, global_key, global_value), bf16
        [B,H,L,64] buffers holding positions [0, row); the new rows are written there
        first. Every sequence is row + T long, so the router's chunk representatives
        are rebuilt at that length and only the selector tiles holding the new rows
        are selected, routed and attended (a partially filled tile is selected from
        its present queries, exactly as a prefill of row + T tokens selects it).
        Returns (W_o(attended) [B,T,D], content-gate logits [B,T,D]).
        """
        self._check_supported()
        B, T, _ = x.shape
        act = torch.bfloat16
        xb = x if x.dtype == act else x.to(act)
        qkvg, down = self._project(xb)
        q, k, v, gate = qkvg.split(self.D, dim=-1)
        query = _to_heads(q, B, T, self.H, self.hd)
        local_key = _to_heads(k, B, T, self.H, self.hd)
        local_value = _to_heads(v, B, T, self.H, self.hd)
        global_key, global_value = self.global_kv(xb, local_key, local_value, kv_inject, down)
        seq_len = row + T
        if seq_len > cache[0].shape[2]:
            raise ValueError(f"rows [{row}, {seq_len}) exceed the cache length {cache[0].shape[2]}")
        for buf, new in zip(cache, (query, local_key, local_value, global_key, global_value)):
            buf[:, :, row:seq_len].copy_(new)
        cq, clk, clv, cgk, cgv = (buf[:, :, :seq_len] for buf in cache)
        lengths = torch.full((B,), seq_len, dtype=torch.int32, device=x.device)
        tile0 = row // _TILE
        tiles = -(-seq_len // _TILE) - tile0
        reps = chunk_representatives(cgk, lengths, blend_alpha=self._blend_alpha)
        top, _ = select_chunks(cq, reps, lengths, top_k=self.top_k_chunks, temperature=self.temperature,
                               tile_begin=tile0, tile_count=tiles)
        scale = self.route_prior_scale.detach().float().contiguous()
        attended = torch.empty(B, seq_len, self.D, dtype=act, device=x.device)
        tile_attention(cq, clk, clv, cgk, cgv, reps, top, scale, lengths,
                       out=_to_heads(attended, B, seq_len, self.H, self.hd), tile_begin=tile0, tile_count=tiles)
        return gemm.linear(attended[:, row:], self.W_o.weight.to(act)), gate

    def forward_step(self, x: torch.Tensor, kv_inject, cache, reps: torch.Tensor, attended: torch.Tensor,
                     pos: torch.Tensor, lengths: torch.Tensor):
        """``forward_parts_cached`` for one new token per sequence at the device position
        ``pos`` (int64 [1]); every launch takes the position from device memory, so the step
        can be captured once in a CUDA graph and replayed at every position.

        ``reps`` [B,H,L/64,64] holds the chunk representatives of the cached positions
        (only the chunk holding ``pos`` changes), ``attended`` [B,L,D] is scratch and
        ``lengths`` int32 [B] = pos + 1. Returns (W_o(attended) [B,1,D], gate logits).
        """
        self._check_supported()
        B = x.shape[0]
        act = torch.bfloat16
        xb = x if x.dtype == act else x.to(act)
        qkvg, down = self._project(xb)
        q, k, v, gate = qkvg.split(self.D, dim=-1)
        query = _to_heads(q, B, 1, self.H, self.hd)
        local_key = _to_heads(k, B, 1, self.H, self.hd)
        local_value = _to_heads(v, B, 1, self.H, self.hd)
        global_key, global_value = self.global_kv(xb, local_key, local_value, kv_inject, down)
        for buf, new in zip(cache, (query, local_key, local_value, global_key, global_value)):
            buf.index_copy_(2, pos, new)
        cq, clk, clv, cgk, cgv = cache
        L = cq.shape[2]
        chunk_representatives(cgk, lengths, blend_alpha=self._blend_alpha, out=reps, pos=pos)
        top, _ = select_chunks(cq, reps, lengths, top_k=self.top_k_chunks, temperature=self.temperature,
                               tile_count=1, pos=pos)
        scale = self.route_prior_scale.detach().float().contiguous()
        tile_attention(cq, clk, clv, cgk, cgv, reps, top, scale, lengths,
                       out=_to_heads(attended, B, L, self.H, self.hd), tile_count=1, pos=pos)
        return gemm.linear(attended.index_select(1, pos), self.W_o.weight.to(act)), gate

    def _forward_autograd(self, x: torch.Tensor, kv_inject, lengths: torch.Tensor, *,
                          router_inputs: list | None = None):
        """Differentiable forward (training, or any call that needs gradients): the
        reference forward (hierarchical_sparse_attn_v18_hisa.py:2546-2787) with the
        projections, the global adapters, the NPCI rotation, the chunk representatives,
        the route prior and the router's auxiliary loss as torch ops on the device, the
        chunk selection on ``dwarf_hisa_select`` (plus the training-mode exploration
        slot) and the attention on ``dwarf_hisa_attn`` / ``dwarf_hisa_attn_bwd``.
        Returns (output [B,T,D] in x's dtype, top_chunk_idx, auxiliary loss)."""
        B, T, _ = x.shape
        q, k, v, gate = self.qkvg_proj(x).split(self.D, dim=-1)
        query = _to_heads(q, B, T, self.H, self.hd)
        local_key = _to_heads(k, B, T, self.H, self.hd)
        local_value = _to_heads(v, B, T, self.H, self.hd)
        global_key, global_value = local_key, local_value
        if self.global_adapter_rank:
            global_key = global_key + _to_heads(self.global_k_up(self.global_k_down(x)), B, T, self.H, self.hd)
            global_value = global_value + _to_heads(self.global_v_up(self.global_v_down(x)), B, T, self.H, self.hd)
        if kv_inject is not None:
            kd, vd = kv_inject
            if kd.shape != global_key.shape or vd.shape != global_value.shape:
                raise ValueError("kv_inject must contain [B,H,N,HD] tensors")
            global_key = npci_rotate_autograd(global_key, kd, self.npci_theta_max * torch.tanh(self.npci_theta_k))
            global_value = npci_rotate_autograd(global_value, vd,
                                                self.npci_theta_max * torch.tanh(self.npci_theta_v))
        reps = representatives_autograd(global_key, lengths, self._blend_alpha)
        query_normalized = F.normalize(query.float(), dim=-1, eps=1e-6).to(query.dtype)
        tiles = -(-T // self.selector_tile_size)
        starts = (torch.arange(tiles, device=x.device) * self.selector_tile_size).clamp_max(T - 1)
        anchor = query_normalized[:, :, starts]
        anchor_logits = torch.matmul(anchor.float(), reps.float().transpose(-2, -1)) / self.temperature
        act = torch.bfloat16
        top, _ = select_chunks(query.detach().to(act).contiguous(), reps.detach().to(act).contiguous(), lengths,
                               top_k=self.top_k_chunks, temperature=self.temperature)
        if router_inputs is not None:
            router_inputs.extend((query.detach(), global_key.detach()))
        if self.training and self.exploration_probability > 0.0:
            top = inject_exploration(top, _eligible(tiles, reps.shape[2], lengths), self.exploration_probability)
        route = selected_route_scores(query_normalized, reps, top, self.route_prior_scale)
        auxiliary = None
        if self.training and self.route_aux_weight > 0.0:
            auxiliary = router_auxiliary_loss(anchor_logits, anchor, global_key, lengths,
                                              samples=self.route_aux_samples,
                                              temperature=self.route_aux_temperature) * self.route_aux_weight
            self._routing_auxiliary_loss = auxiliary
            self.hisa_evidence_capture = HISASelectionCapture(anchor_logits=anchor_logits,
                                                              metadata=self._metadata(top, lengths),
                                                              auxiliary_loss=auxiliary)
        self._last_token_selection_path = "enumerate_all"
        attended = hisa_tile_attention(query, local_key, local_value, global_key, global_value, route, top, lengths)
        merged = attended.to(x.dtype).permute(0, 2, 1, 3).reshape(B, T, self.D)
        output = self.W_o(merged) * torch.sigmoid(gate)
        if auxiliary is None:
            auxiliary = output.sum() * 0.0
        return output, top, auxiliary

    def _canonical_metadata(self, query: torch.Tensor, global_key: torch.Tensor, top: torch.Tensor,
                            lengths: torch.Tensor) -> HISAMetadata:
        """The metadata the reference returns when asked for it: the routed chunks and, per
        (tile, slot), the chunk's tokens in descending order of the tile anchor's score
        q^_anchor . k / sqrt(hd), invalid tokens (past the valid length, at or after the
        tile start, or of an empty slot) as -1 / -inf (reference
        _build_causal_tile_metadata with canonical_token_order, :290-397; the module
        asks for it whenever return_metadata is set, :2625). The attention does not
        depend on this listing: with top_m_tokens == chunk_size every valid token of a
        routed chunk is attended either way."""
        with torch.no_grad():
            B, H, T, D = query.shape
            tiles, k_slots = top.shape[2], top.shape[3]
            chunk = self.chunk_size
            starts = torch.arange(tiles, device=query.device, dtype=torch.int32) * self.selector_tile_size
            qn = F.normalize(query.float(), dim=-1, eps=1e-6).to(query.dtype)
            anchor = qn[:, :, starts.long().clamp_max(T - 1)]
            chunks = -(-T // chunk)
            keys = F.pad(global_key, (0, 0, 0, chunks * chunk - T)).reshape(B, H, chunks, chunk, D)
            bi = torch.arange(B, device=query.device).view(B, 1, 1, 1)
            hi = torch.arange(H, device=query.device).view(1, H, 1, 1)
            picked = keys[bi, hi, top.clamp_min(0).long()]                       # [B,H,tiles,K,chunk,D]
            within = torch.arange(chunk, device=query.device, dtype=torch.int32).view(1, 1, 1, 1, chunk)
            absolute = top[..., None] * chunk + within
            valid = ((top[..., None] >= 0) & (absolute < lengths.view(B, 1, 1, 1, 1))
                     & (absolute < starts.view(1, 1, tiles, 1, 1)))
            scores = torch.einsum("bhtd,bhtkmd->bhtkm", anchor.float(), picked.float()) / math.sqrt(D)
            scores = scores.masked_fill(~valid, float("-inf"))
            token_scores, local = scores.topk(min(self.hisa_top_m_tokens, chunk), dim=-1)
            finite = torch.isfinite(token_scores) & (top[..., None] >= 0)
            token_idx = torch.where(finite, top[..., None] * chunk + local.to(torch.int32),
                                    torch.full_like(local, -1, dtype=torch.int32)).to(torch.int32)
            token_scores = torch.where(finite, token_scores, torch.full_like(token_scores, float("-inf")))
        return HISAMetadata(top_chunk_idx=top, token_idx=token_idx, token_scores=token_scores.float(),
                            tile_starts=starts, valid_lengths=lengths, chunk_size=self.chunk_size,
                            selector_tile_size=self.selector_tile_size, enumerate_all=False)

    def _metadata(self, top: torch.Tensor, lengths: torch.Tensor) -> HISAMetadata:
        tiles = top.shape[2]
        return HISAMetadata(
            top_chunk_idx=top,
            token_idx=torch.empty(0, dtype=torch.int32, device=top.device),
            token_scores=torch.empty(0, dtype=torch.float32, device=top.device),
            tile_starts=torch.arange(tiles, device=top.device, dtype=torch.int32) * self.selector_tile_size,
            valid_lengths=lengths, chunk_size=self.chunk_size, selector_tile_size=self.selector_tile_size,
            enumerate_all=True)

    def forward(self, x: torch.Tensor, kv_inject=None, *, valid_lengths=None, return_metadata: bool = False,
                return_auxiliary: bool = False):
        self._check_supported()
        _lib.require_cuda(x)
        self.hisa_evidence_capture = None
        self._routing_auxiliary_loss = None
        B, T, _ = x.shape
        if -(-T // self.chunk_size) > 128:
            raise ValueError("the B200 HISA router supports up to 128 chunks (T <= 8192)")
        lengths = _as_valid_lengths(
            valid_lengths if valid_lengths is not None else getattr(self, "_causal_control_valid_lengths", None),
            batch_size=B, seq_len=T, device=x.device)
        grad = torch.is_grad_enabled() and (x.requires_grad or any(p.requires_grad for p in self.parameters()))
        router_inputs: list = []
        if grad or self.training:
            output, top, auxiliary = self._forward_autograd(x, kv_inject, lengths, router_inputs=router_inputs)
        else:
            projected, gate, top = self.forward_parts(x, kv_inject, lengths,
                                                      router_inputs=router_inputs if return_metadata else None)
            output = gate_mul(projected, gate)
            if x.dtype != torch.bfloat16:
                output = output.to(x.dtype)
            auxiliary = output.new_zeros(())
        if return_metadata:
            metadata = self._canonical_metadata(*router_inputs, top, lengths)
            return (output, metadata, auxiliary) if return_auxiliary else (output, metadata)
        return (output, auxiliary) if return_auxiliary else output


HierarchicalSparseAttentionV17HISACausal = HierarchicalSparseAttentionV16HISACausal
HierarchicalSparseAttentionV18HISACausal = HierarchicalSparseAttentionV16HISACausal
