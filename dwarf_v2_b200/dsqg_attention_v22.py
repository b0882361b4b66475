"""DSQG lattice attention on B200: drop-in for the reference ``kernels/dsqg_attention_v22.py``.

Public surface kept from the reference (same names, arguments, validation
errors and state_dict layout):

* constants ``ALL_OFFSETS`` (:84-94), ``R_PLANES``, ``NPCI_THETA_MAX``,
  ``NPCI_THETA_INIT``, ``GROUPED_MODE_IDS``;
* ``dsqg_attention_v18_grouped(q, k, v, ..., plane_shift=0, query_start=0, *,
  backend="auto", online_softmax=True)`` (:2691-2777);
* ``DSQGAttentionV19`` (aliases V20/V21/V22) with ``forward(x, kv_inject=None)``
  (:2788-3289), ``pos_bias``, ``centered_scale_embed``, ``semantic_config``,
  ``execution_config``, ``support_statistics``, ``phase_probe_regularizer``;
* helpers ``npci_rotate``, ``calibrated_movt_phase_gain_std``.

Engine additions: ``dsqg_attention_q6`` (DSQG over a q6 KV cache) and the
module option ``kv_cache="q6"``.

Everything on the device runs in this engine's CUDA kernels (``dwarf_dsqg_prep``,
``dwarf_dsqg_fwd``, ``dwarf_npci_rotate``) and its tcgen05 GEMM (``dwarf_gemm_bf16``); there is no
Triton, no eager fallback and no CPU path (CPU tensors raise). Every grouped
mode computes the same function, so all of them run the one online kernel.
"""

from __future__ import annotations

import math
import os

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib, gemm
from .npci import npci_rotate_autograd, npci_rotate_cuda

R_PLANES = 4
NPCI_THETA_MAX = 0.25
NPCI_THETA_INIT = 0.01

# The canonical 96-offset DSQG lattice. The table is data that must be
# identical to the reference's (kernels/dsqg_attention_v22.py:84-94).
ALL_OFFSETS = [
    1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 13, 15, 16, 19, 21, 23, 28,
    48, 64, 96, 121, 161, 192, 212, 245, 273, 295, 342, 375, 384,
    413, 441, 473, 512, 549, 579, 593, 631, 653, 694, 716, 768,
    826, 846, 900, 936, 970, 1000, 1024, 1074, 1108, 1144, 1166,
    1190, 1218, 1244, 1288, 1322, 1385, 1423, 1451, 1497, 1522,
    1550, 1581, 1603, 1617, 1634, 1651, 1661, 1710, 1743, 1780,
    1810, 1820, 1852, 1860, 1876, 1886, 1897, 1903, 1916, 1926,
    1929, 1941, 1965, 1983, 2006, 2011, 2029, 2037, 2044, 2068,
    2097, 2113, 2199,
]

GROUPED_MODE_IDS = {"baseline": 0, "overlap_slab": 1, "overlap_slab_bwd": 3}
_UNIMPLEMENTED_GROUPED_MODES = {"packed_kv"}
SMALL_BAND_MAX = 28  # offsets <= 28 form the dense band
LARGE_BAND_MIN = 48  # offsets >= 48 form the sparse band (MOVT-rotated values)


# --------------------------------------------------------------------------- config helpers

def _as_int(name: str, value, *, minimum: int) -> int:
    """Integer argument without bool/float coercion (reference :482-494)."""
    if isinstance(value, bool) or not hasattr(value, "__index__"):
        raise TypeError(f"{name} must be an integer >= {minimum}, got {type(value).__name__}")
    ivalue = int(value.__index__())
    if ivalue < minimum:
        raise ValueError(f"{name}={ivalue} must be >= {minimum}")
    return ivalue


_normalize_int_arg = _as_int


def _next_pow2(n: int) -> int:
    return 1 if n <= 1 else 1 << (int(n) - 1).bit_length()


def _env_float(name: str, default: float) -> float:
    raw = os.environ.get(name)
    if raw is None or str(raw).strip() == "":
        return float(default)
    try:
        return float(raw)
    except ValueError as exc:
        raise ValueError(f"{name} must be a float, got {raw!r}") from exc


def _normalize_plane_shift(r_planes: int, hd: int, plane_shift: int = 0) -> int:
    """Validate the MOVT channel-pair shift (reference :109-128)."""
    if isinstance(plane_shift, bool):
        raise TypeError("plane_shift must be an integer, got bool")
    if not hasattr(plane_shift, "__index__"):
        raise TypeError(f"plane_shift must be an integer, got {type(plane_shift).__name__}")
    shift = int(plane_shift.__index__())
    if hd < 2 * r_planes:
        raise ValueError(f"head_dim={hd} must be >= 2*r_planes={2 * r_planes}")
    segment = max(2, hd // r_planes)
    if not 0 <= shift <= segment - 2:
        raise ValueError(
            f"plane_shift={shift} must keep each MOVT pair inside its hd/r segment; "
            f"allowed range is [0, {segment - 2}] for head_dim={hd}, r_planes={r_planes}"
        )
    return shift


def _phase_plane_channels(r_planes: int, hd: int, plane_shift: int = 0) -> list[tuple[int, int]]:
    """Channel pair of each MOVT plane: (r*hd/R + shift, +1) (reference :131-154)."""
    shift = _normalize_plane_shift(r_planes, hd, plane_shift)
    stride = max(2, hd // r_planes)
    pairs: list[tuple[int, int]] = []
    taken: set[int] = set()
    for r in range(r_planes):
        a = min(r * stride + shift, hd - 2)
        if a in taken or a + 1 in taken:
            free = [c for c in range(hd - 1) if c not in taken and c + 1 not in taken]
            if not free:
                raise ValueError(f"Could not assign {r_planes} disjoint MOVT planes in head_dim={hd}")
            a = free[0]
        taken.update((a, a + 1))
        pairs.append((a, a + 1))
    return pairs


def _canonicalize_offsets(offsets, j_small: int, j_large: int) -> tuple[list[int], int, int]:
    """Sort offsets into [small band | large band] and check the declared sizes (reference :157-186)."""
    values = []
    for d in offsets:
        if isinstance(d, bool):
            raise TypeError(f"DSQG offsets must be integer positive causal deltas, got bool: {d!r}")
        if not hasattr(d, "__index__"):
            raise TypeError(
                f"DSQG offsets must be integer positive causal deltas, got {type(d).__name__}: {d!r}"
            )
        value = int(d.__index__())
        if value <= 0:
            raise ValueError(f"DSQG offsets must be positive causal deltas; got {value}")
        values.append(value)
    if len(set(values)) != len(values):
        raise ValueError(f"Duplicate DSQG offsets are not supported: {values}")
    middle = [d for d in values if SMALL_BAND_MAX < d < LARGE_BAND_MIN]
    if middle:
        raise ValueError(f"Offsets must be <=28 or >=48 for the DSQG split; got middle offsets {middle}")
    small = sorted(d for d in values if d <= SMALL_BAND_MAX)
    large = sorted(d for d in values if d >= LARGE_BAND_MIN)
    if len(small) != int(j_small) or len(large) != int(j_large):
        raise ValueError(
            f"j_small/j_large mismatch after canonicalization: "
            f"declared ({j_small}, {j_large}) vs actual ({len(small)}, {len(large)})"
        )
    return small + large, len(small), len(large)


def calibrated_movt_phase_gain_std(*, head_dim: int, target_dynamic_rms: float, gate_logit: float = 0.0) -> float:
    """Phase-gain std giving the target initial content-angle RMS (reference :196-220)."""
    head_dim, target, gate_logit = int(head_dim), float(target_dynamic_rms), float(gate_logit)
    if head_dim <= 0:
        raise ValueError(f"head_dim must be positive, got {head_dim}")
    if not math.isfinite(target) or target <= 0.0:
        raise ValueError(f"target_dynamic_rms must be finite and positive, got {target_dynamic_rms}")
    if not math.isfinite(gate_logit):
        raise ValueError(f"gate_logit must be finite, got {gate_logit}")
    return target * head_dim * (1.0 + math.exp(-gate_logit))


def npci_rotate(x: torch.Tensor, x_delta: torch.Tensor, theta_h: torch.Tensor, *,
                strength_tau: float = 0.25) -> torch.Tensor:
    """Magnitude-aware norm-preserving rotation of x[B,H,N,D] toward x_delta (reference :223-254)."""
    return npci_rotate_cuda(x, x_delta, theta_h, strength_tau=strength_tau)


def _orthogonal_phase_probes(r_planes: int, hd: int, plane_shift: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """Unit q/k probes on each plane's channel pair, k a quarter turn ahead (reference :257-271)."""
    q = torch.zeros(r_planes, hd, dtype=torch.float32)
    k = torch.zeros(r_planes, hd, dtype=torch.float32)
    for r, (a, b) in enumerate(_phase_plane_channels(r_planes, hd, plane_shift)):
        phi = 2.0 * math.pi * r / max(r_planes, 1)
        q[r, a], q[r, b] = math.cos(phi), math.sin(phi)
        k[r, a], k[r, b] = math.cos(phi + math.pi / 2.0), math.sin(phi + math.pi / 2.0)
    return q, k


def _raw_npci_theta_from_effective(theta: float) -> float:
    theta, limit = float(theta), float(NPCI_THETA_MAX)
    if not 0.0 <= abs(theta) < limit:
        raise ValueError(f"NPCI_THETA_INIT={theta} must satisfy abs(theta) < {limit}")
    return math.atanh(theta / limit)


def _resolve_grouped_mode(mode: str) -> int:
    if not isinstance(mode, str):
        raise TypeError(f"grouped_mode must be a string, got {type(mode).__name__}")
    if mode in _UNIMPLEMENTED_GROUPED_MODES:
        raise NotImplementedError(
            f"grouped_mode='{mode}' is advertised by older configs but is not implemented in this kernel"
        )
    if mode not in GROUPED_MODE_IDS:
        raise ValueError(f"Unknown grouped_mode='{mode}'. Allowed: {', '.join(sorted(GROUPED_MODE_IDS))}")
    return GROUPED_MODE_IDS[mode]


def _normalize_grouping_args(k_group_size, max_group_size, max_group_spread, grouped_mode_id=None):
    """Validate the sparse-grouping knobs (reference :497-535)."""
    k_group_size = _as_int("k_group_size", k_group_size, minimum=1)
    if max_group_size is None:
        max_group_size = k_group_size
    else:
        max_group_size = _as_int("max_group_size", max_group_size, minimum=1)
        if max_group_size > k_group_size:
            raise ValueError(
                f"max_group_size={max_group_size} cannot exceed k_group_size={k_group_size}; "
                "overlap-slab kernels iterate only K_GROUP_SIZE slots per group"
            )
    if grouped_mode_id in (GROUPED_MODE_IDS["overlap_slab"], GROUPED_MODE_IDS["overlap_slab_bwd"]) and (
        max_group_spread is None
    ):
        max_group_spread = 64
    if max_group_spread is not None:
        max_group_spread = _as_int("max_group_spread", max_group_spread, minimum=0)
    return k_group_size, max_group_size, max_group_spread


def _plan_sparse_groups(offsets, j_small, k_group_size, max_group_size=None, max_group_spread=None,
                        slab_block_n: int = 64) -> dict:
    """Group the sorted large-band offsets, minimising sum(slab_block_n + spread).

    Schedule metadata only (the grouping never changes results); it fills the
    reference module's planner buffers (reference :538-672): a shortest-path
    over split points of the sorted sparse offsets, groups of at most
    ``max_group_size`` offsets whose spread stays within ``max_group_spread``.
    """
    k_group_size, max_group_size, max_group_spread = _normalize_grouping_args(
        k_group_size, max_group_size, max_group_spread
    )
    sparse = sorted(range(j_small, len(offsets)), key=lambda i: offsets[i])
    n = len(sparse)
    keys = ("sparse_order", "group_start", "group_len", "group_dmin", "group_dmax", "group_i", "group_rel")
    if n == 0:
        return {**{k: [] for k in keys}, "max_group_len": 0, "max_group_spread": 0}
    best = [math.inf] * (n + 1)
    back: list[int | None] = [None] * (n + 1)
    best[0] = 0.0
    for start in range(n):
        if best[start] == math.inf:
            continue
        lo = hi = offsets[sparse[start]]
        for length in range(1, max_group_size + 1):
            end = start + length
            if end > n:
                break
            d = offsets[sparse[end - 1]]
            lo, hi = min(lo, d), max(hi, d)
            if max_group_spread is not None and hi - lo > max_group_spread:
                break
            cost = best[start] + float(slab_block_n) + (hi - lo)
            if cost < best[end]:
                best[end], back[end] = cost, start
    if back[n] is None:
        spans = [(i, min(i + max_group_size, n)) for i in range(0, n, max_group_size)]
    else:
        spans, end = [], n
        while end > 0:
            start = back[end]
            spans.append((start, end))
            end = start
        spans.reverse()
    plan = {k: [] for k in keys}
    cursor = max_len = max_spread = 0
    for start, end in spans:
        idxs = sparse[start:end]
        deltas = [offsets[i] for i in idxs]
        plan["sparse_order"].extend(idxs)
        plan["group_start"].append(cursor)
        plan["group_len"].append(len(idxs))
        plan["group_dmin"].append(min(deltas))
        plan["group_dmax"].append(max(deltas))
        plan["group_i"].append(idxs)
        plan["group_rel"].append([max(deltas) - d for d in deltas])
        max_len = max(max_len, len(idxs))
        max_spread = max(max_spread, max(deltas) - min(deltas))
        cursor += len(idxs)
    plan["max_group_len"] = max_len
    plan["max_group_spread"] = max_spread
    return plan


def _verify_sparse_plan(offsets, j_small: int, plan: dict) -> None:
    if sorted(plan["sparse_order"]) != list(range(j_small, len(offsets))):
        raise AssertionError("Sparse plan does not include each sparse logical index exactly once")
    for gi, start in enumerate(plan["group_start"]):
        dmax = plan["group_dmax"][gi]
        for t in range(plan["group_len"][gi]):
            idx = plan["sparse_order"][start + t]
            rel = plan["group_rel"][gi][t]
            if rel != dmax - offsets[idx]:
                raise AssertionError(
                    f"Invalid rel mapping at group={gi}, t={t}: rel={rel}, dmax={dmax}, delta={offsets[idx]}"
                )


# --------------------------------------------------------------------------- kernel entry points

def _strides3(t: torch.Tensor) -> tuple[int, int, int]:
    return t.stride(0), t.stride(1), t.stride(2)


def _dsqg_launch(q, *, kv, pos_bias, scale_embed, phase_base, phase_gain, y_pre, z_pre, offsets,
                 j_small, j_large, plane_shift, query_start, out, lse=None, head_gain=None, gate=None,
                 seq_len=None, row_begin=0, pos=None):
    """Validate and launch dwarf_dsqg_fwd. ``kv`` is ("bf16", k, v) or ("q6", kc, ks, vc, vs).

    With ``row_begin`` > 0 only queries [row_begin, seq_len) are computed and q, y_pre,
    gate, out and lse hold those rows only (row 0 = position row_begin); K/V and z_pre
    cover positions [0, seq_len). This is the decode step's single-row launch.
    ``pos`` (device int64 [1]) instead supplies row_begin at run time (a decode step
    replayed from a CUDA graph); y_pre rows are then absolute positions like z_pre's.
    """
    B, H, N, HD = q.shape
    if seq_len is not None:
        N = int(seq_len)
    J = int(j_small) + int(j_large)
    if HD != 64:
        raise ValueError(f"the B200 DSQG kernel supports head_dim 64, got {HD}")
    args = _lib.DsqgFwdArgs(version=_lib.ABI_VERSION, B=B, H=H, N=N, head_dim=HD, J=J,
                            j_small=int(j_small), j_large=int(j_large), plane_shift=int(plane_shift),
                            query_start=int(query_start), row_begin=int(row_begin))
    args.q = q.data_ptr()
    args.sqb, args.sqh, args.sqn = _strides3(q)
    if kv[0] == "bf16":
        _, k, v = kv
        args.kv_format = 0
        args.H_kv = k.shape[1]
        args.k, args.v = k.data_ptr(), v.data_ptr()
        args.skb, args.skh, args.skn = _strides3(k)
        args.svb, args.svh, args.svn = _strides3(v)
    else:
        _, kc, ks, vc, vs = kv
        args.kv_format = 1
        args.H_kv = kc.shape[1]
        args.k_codes, args.k_scales = kc.data_ptr(), ks.data_ptr()
        args.v_codes, args.v_scales = vc.data_ptr(), vs.data_ptr()
        args.ccb, args.cch, args.cct = _strides3(kc)
        args.csb, args.csh, args.cst = _strides3(ks)
    args.offsets = offsets.data_ptr()
    args.pos_bias, args.spj, args.sph = pos_bias.data_ptr(), pos_bias.stride(0), pos_bias.stride(1)
    args.scale_embed, args.sej, args.sed = scale_embed.data_ptr(), scale_embed.stride(0), scale_embed.stride(1)
    args.phase_base, args.sbj, args.sbh = phase_base.data_ptr(), phase_base.stride(0), phase_base.stride(1)
    args.phase_gain, args.sgj, args.sgh = phase_gain.data_ptr(), phase_gain.stride(0), phase_gain.stride(1)
    args.y_pre = y_pre.data_ptr()
    args.syb, args.syh, args.syn = _strides3(y_pre)
    args.z_pre = z_pre.data_ptr()
    args.szb, args.szh, args.szn = _strides3(z_pre)
    args.out = out.data_ptr()
    args.sob, args.soh, args.son = _strides3(out)
    if lse is not None:
        args.lse = lse.data_ptr()
        args.slb, args.slh, args.sln = _strides3(lse)
    if head_gain is not None:
        args.head_gain = head_gain.data_ptr()
        args.head_gain_dtype = _lib.dtype_code(head_gain.dtype)
    if gate is not None:
        args.gate = gate.data_ptr()
        args.sgb_, args.sgn_ = gate.stride(0), gate.stride(1)
    if pos is not None:
        args.pos = pos.data_ptr()
    _lib.call("dwarf_dsqg_fwd", args, q.device)


def _prepare_tables(pos_bias, scale_embed, phase_base, phase_gain, y_pre, z_pre, offsets_dev, device, J, j_large):
    def f32(t):
        return t.detach().to(device=device, dtype=torch.float32).contiguous()

    pb, se = f32(pos_bias), f32(scale_embed)
    if pb.shape != (J, pb.shape[1]) or se.shape != (J, 64):
        raise ValueError(f"pos_bias must be [J,H] and scale_embed [J,64] with J={J}")
    pbase, pgain = f32(phase_base), f32(phase_gain)
    if j_large > 0 and (pbase.shape[0] < j_large or pbase.shape[-1] != R_PLANES):
        raise ValueError("phase_base/phase_gain must be [j_large,H,4]")
    offsets = offsets_dev.detach().to(device=device, dtype=torch.int32).contiguous()
    if offsets.numel() != J:
        raise ValueError(f"offsets must hold J={J} entries")
    return pb, se, pbase, pgain, f32(y_pre), f32(z_pre), offsets


def _check_common(q, k, v, y_pre, z_pre):
    B, H, N, HD = q.shape
    Bk, H_kv, Nk, HDk = k.shape
    if v.shape != k.shape:
        raise ValueError(f"k/v shape mismatch: k={tuple(k.shape)} v={tuple(v.shape)}")
    if Bk != B or Nk != N or HDk != HD:
        raise ValueError(f"native GQA requires q/k/v to share B,N,HD: q={tuple(q.shape)} k={tuple(k.shape)}")
    if H % H_kv != 0:
        raise ValueError(f"num query heads H={H} must be divisible by KV heads H_KV={H_kv}")
    if tuple(y_pre.shape[:3]) != (B, H, N):
        raise ValueError(f"y_pre must have shape [B,Hq,N,R]; got {tuple(y_pre.shape)} for q={tuple(q.shape)}")
    if tuple(z_pre.shape[:3]) != (B, H_kv, N):
        raise ValueError(f"z_pre must have shape [B,Hkv,N,R]; got {tuple(z_pre.shape)} for k={tuple(k.shape)}")


def _forward_only(*tensors) -> None:
    if torch.is_grad_enabled() and any(isinstance(t, torch.Tensor) and t.requires_grad for t in tensors):
        raise NotImplementedError("dwarf_v2_b200 is a forward (inference) engine; run under torch.no_grad()")


def _needs_grad(*tensors) -> bool:
    return torch.is_grad_enabled() and any(isinstance(t, torch.Tensor) and t.requires_grad for t in tensors)


class _DSQGFn(torch.autograd.Function):
    """Differentiable DSQG over bf16 K/V (reference _DSQGV18GroupedFn,
    dsqg_attention_v22.py:2197-2552): forward by ``dwarf_dsqg_fwd`` (which also
    writes the natural-log lse), backward by ``dwarf_dsqg_bwd`` (dq, dk, dv,
    dy_pre, dz_pre, phase-table gradients and the per-pair ds), then
    d pos_bias = sum_{b,n} ds and d scale_embed = (1/8) sum ds q."""

    @staticmethod
    def forward(ctx, q, k, v, pos_bias, scale_embed, phase_base, phase_gain, y_pre, z_pre,
                offsets, j_small, j_large, plane_shift, query_start):
        B, H, N, HD = q.shape
        qb, kb, vb = (t.to(torch.bfloat16).contiguous() for t in (q, k, v))
        J = int(j_small) + int(j_large)
        pb, se, pbase, pgain, y32, z32, offs = _prepare_tables(
            pos_bias, scale_embed, phase_base, phase_gain, y_pre, z_pre, offsets, q.device, J, int(j_large))
        out = torch.empty(B, H, N, HD, dtype=torch.bfloat16, device=q.device)
        lse = torch.empty(B, H, N, dtype=torch.float32, device=q.device)
        _dsqg_launch(qb, kv=("bf16", kb, vb), pos_bias=pb, scale_embed=se, phase_base=pbase, phase_gain=pgain,
                     y_pre=y32, z_pre=z32, offsets=offs, j_small=j_small, j_large=j_large,
                     plane_shift=plane_shift, query_start=query_start, out=out, lse=lse)
        ctx.save_for_backward(qb, kb, vb, out, lse, pb, se, pbase, pgain, y32, z32, offs)
        ctx.meta = (int(j_small), int(j_large), int(plane_shift), int(query_start))
        ctx.in_dtypes = tuple(t.dtype for t in (q, k, v, pos_bias, scale_embed, phase_base, phase_gain,
                                                  y_pre, z_pre))
        ctx.phase_shape = tuple(phase_base.shape)
        return out if q.dtype == torch.bfloat16 else out.to(q.dtype)

    @staticmethod
    def backward(ctx, dout):
        qb, kb, vb, out, lse, pb, se, pbase, pgain, y32, z32, offs = ctx.saved_tensors
        j_small, j_large, plane_shift, query_start = ctx.meta
        B, H, N, HD = qb.shape
        H_kv = kb.shape[1]
        J = j_small + j_large
        dev = qb.device
        dob = dout.to(torch.bfloat16).contiguous()
        dq, dk, dv = torch.empty_like(qb), torch.empty_like(kb), torch.empty_like(vb)
        dy, dz = torch.empty_like(y32), torch.empty_like(z32)
        ds = torch.zeros(B, H, N, J, dtype=torch.float32, device=dev)
        delta = torch.empty(B, H, N, dtype=torch.float32, device=dev)
        dpbase = torch.zeros(max(j_large, 1), H, 4, dtype=torch.float32, device=dev)
        dpgain = torch.zeros_like(dpbase)
        pbase_c = pbase[:j_large].contiguous()
        pgain_c = pgain[:j_large].contiguous()
        args = _lib.DsqgBwdArgs(version=_lib.ABI_VERSION, J=J, j_small=j_small, j_large=j_large,
                                plane_shift=plane_shift, query_start=query_start, B=B, H=H, H_kv=H_kv, N=N)
        for name, t in (("q", qb), ("k", kb), ("v", vb), ("out", out), ("dout", dob), ("lse", lse),
                        ("offsets", offs), ("pos_bias", pb), ("scale_embed", se), ("phase_base", pbase_c),
                        ("phase_gain", pgain_c), ("y_pre", y32), ("z_pre", z32), ("dq", dq), ("dk", dk),
                        ("dv", dv), ("dy_pre", dy), ("dz_pre", dz), ("ds", ds), ("delta", delta),
                        ("d_phase_base", dpbase), ("d_phase_gain", dpgain)):
            setattr(args, name, t.data_ptr())
        _lib.call("dwarf_dsqg_bwd", args, dev)
        d_pos_bias = ds.sum(dim=(0, 2)).transpose(0, 1)
        d_scale_embed = torch.einsum("bhnj,bhnd->jd", ds, qb.float()) * 0.125
        (q_dt, k_dt, v_dt, pb_dt, se_dt, pbase_dt, pgain_dt, y_dt, z_dt) = ctx.in_dtypes
        d_pbase = torch.zeros(ctx.phase_shape, dtype=torch.float32, device=dev)
        d_pgain = torch.zeros_like(d_pbase)
        if j_large > 0:
            d_pbase[:j_large] = dpbase
            d_pgain[:j_large] = dpgain
        return (dq.to(q_dt), dk.to(k_dt), dv.to(v_dt), d_pos_bias.to(pb_dt), d_scale_embed.to(se_dt),
                d_pbase.to(pbase_dt), d_pgain.to(pgain_dt), dy.to(y_dt), dz.to(z_dt),
                None, None, None, None, None)


def _bf16_rows(t: torch.Tensor) -> torch.Tensor:
    """bf16 view usable by the kernels: dim stride 1 and 16-byte aligned rows."""
    t = t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)
    ok = t.stride(-1) == 1 and all(s % 8 == 0 for s in t.stride()[:-1]) and t.data_ptr() % 16 == 0
    return t if ok else t.contiguous()


def dsqg_attention_v18_grouped(
    q, k, v, pos_bias, scale_embed, phase_base, phase_gain, y_pre, z_pre,
    j_val, j_small, j_large, offsets_dev, sparse_order_dev, group_start_dev, group_len_dev,
    group_dmin_dev, group_dmax_dev, k_group_size, grouped_mode_id, verify_mode,
    max_group_spread_observed, plane_shift=0, query_start=0, *, backend: str = "auto",
    online_softmax: bool = True,
):
    """DSQG forward over bf16 K/V (reference :2691-2777), run by ``dwarf_dsqg_fwd``.

    The grouping/planner arguments and ``online_softmax`` are accepted for
    signature compatibility; they only select schedules of the same function
    in the reference, and this engine has one schedule.
    """
    del sparse_order_dev, group_start_dev, group_len_dev, group_dmin_dev, group_dmax_dev
    del k_group_size, grouped_mode_id, verify_mode, max_group_spread_observed, online_softmax
    backend = str(backend).lower()
    if backend not in {"auto", "triton", "eager", "cuda"}:
        raise ValueError("backend must be auto, triton, or eager")
    if backend == "eager":
        raise NotImplementedError("the B200 engine has no eager backend; use backend='auto'")
    _lib.require_cuda(q, k, v)
    _check_common(q, k, v, y_pre, z_pre)
    if int(j_val) != int(j_small) + int(j_large):
        raise ValueError("j_val must equal j_small + j_large")
    B, H, N, HD = q.shape
    query_start = max(0, min(int(query_start), N))
    if _needs_grad(q, k, v, pos_bias, scale_embed, phase_base, phase_gain, y_pre, z_pre):
        if HD != 64:
            raise ValueError(f"the B200 DSQG kernel supports head_dim 64, got {HD}")
        if not 0 <= int(plane_shift) <= 14:
            raise ValueError("plane_shift must be in [0, 14] for the backward kernel")
        return _DSQGFn.apply(q, k, v, pos_bias, scale_embed, phase_base, phase_gain, y_pre, z_pre,
                             offsets_dev, int(j_small), int(j_large), int(plane_shift), query_start)
    original_dtype = q.dtype
    qb, kb, vb = _bf16_rows(q), _bf16_rows(k), _bf16_rows(v)
    pb, se, pbase, pgain, y32, z32, offsets = _prepare_tables(
        pos_bias, scale_embed, phase_base, phase_gain, y_pre, z_pre, offsets_dev, q.device, int(j_val), int(j_large)
    )
    out = torch.empty(B, H, N, HD, dtype=torch.bfloat16, device=q.device)
    _dsqg_launch(qb, kv=("bf16", kb, vb), pos_bias=pb, scale_embed=se, phase_base=pbase, phase_gain=pgain,
                 y_pre=y32, z_pre=z32, offsets=offsets, j_small=j_small, j_large=j_large,
                 plane_shift=plane_shift, query_start=query_start, out=out)
    return out if original_dtype == torch.bfloat16 else out.to(original_dtype)


def dsqg_attention_q6(q, k_codes, k_scales, v_codes, v_scales, pos_bias, scale_embed, phase_base, phase_gain,
                      y_pre, z_pre, offsets, j_small, j_large, plane_shift=0, query_start=0,
                      return_lse: bool = False):
    """DSQG forward over a q6 KV cache (codes uint8 [B,Hkv,N,48], scales fp16 [B,Hkv,N])."""
    _lib.require_cuda(q, k_codes, v_codes)
    _forward_only(q)
    B, H, N, HD = q.shape
    if k_codes.shape != v_codes.shape or k_codes.shape[-1] != 48 or k_codes.dtype != torch.uint8:
        raise ValueError("k_codes/v_codes must be uint8 [B,Hkv,N,48] of equal shape")
    if k_scales.shape != k_codes.shape[:3] or v_scales.shape != k_scales.shape:
        raise ValueError("scales must be fp16 [B,Hkv,N]")
    if k_codes.stride() != v_codes.stride() or k_scales.stride() != v_scales.stride():
        raise ValueError("K and V caches must share strides")
    if k_codes.shape[0] != B or k_codes.shape[2] != N or H % k_codes.shape[1]:
        raise ValueError("q and the q6 cache must share B and N, with H divisible by H_kv")
    J = int(j_small) + int(j_large)
    pb, se, pbase, pgain, y32, z32, offs = _prepare_tables(
        pos_bias, scale_embed, phase_base, phase_gain, y_pre, z_pre, offsets, q.device, J, int(j_large)
    )
    qb = _bf16_rows(q)
    out = torch.empty(B, H, N, HD, dtype=torch.bfloat16, device=q.device)
    lse = torch.empty(B, H, N, dtype=torch.float32, device=q.device) if return_lse else None
    _dsqg_launch(qb, kv=("q6", k_codes, k_scales, v_codes, v_scales), pos_bias=pb, scale_embed=se,
                 phase_base=pbase, phase_gain=pgain, y_pre=y32, z_pre=z32, offsets=offs, j_small=j_small,
                 j_large=j_large, plane_shift=plane_shift, query_start=max(0, min(int(query_start), N)),
                 out=out, lse=lse)
    return (out, lse) if return_lse else out


def dsqg_prep(q, k, v, q_probe, k_probe, *, pack_q6: bool):
    """y_pre/z_pre probe projections (+ optional q6 pack of K/V) in one kernel."""
    B, H, N, _ = q.shape
    H_kv = k.shape[1]
    dev = q.device
    y = torch.empty(B, H, N, R_PLANES, dtype=torch.float32, device=dev)
    z = torch.empty(B, H_kv, N, R_PLANES, dtype=torch.float32, device=dev)
    args = _lib.DsqgPrepArgs(version=_lib.ABI_VERSION, pack_q6=int(pack_q6), B=B, H=H, H_kv=H_kv, N=N)
    args.q, (args.sqb, args.sqh, args.sqn) = q.data_ptr(), _strides3(q)
    args.k, (args.skb, args.skh, args.skn) = k.data_ptr(), _strides3(k)
    args.q_probe, args.k_probe = q_probe.data_ptr(), k_probe.data_ptr()
    args.y_pre, args.z_pre = y.data_ptr(), z.data_ptr()
    cache = None
    if pack_q6:
        args.v, (args.svb, args.svh, args.svn) = v.data_ptr(), _strides3(v)
        kc = torch.empty(B, H_kv, N, 48, dtype=torch.uint8, device=dev)
        vc = torch.empty_like(kc)
        ks = torch.empty(B, H_kv, N, dtype=torch.float16, device=dev)
        vs = torch.empty_like(ks)
        args.k_codes, args.k_scales, args.v_codes, args.v_scales = kc.data_ptr(), ks.data_ptr(), vc.data_ptr(), vs.data_ptr()
        cache = (kc, ks, vc, vs)
    _lib.call("dwarf_dsqg_prep", args, dev)
    return y, z, cache


# --------------------------------------------------------------------------- module

class DSQGAttentionV19(nn.Module):
    """DSQG attention block with the reference's parameters and forward contract (reference :2780-3289).

    Forward pipeline on the device. With ``kv_cache="q6"`` (no K/V injection):
    the qkvg GEMM on tcgen05 with the probe projections and the q6 pack of K/V
    fused into its epilogue (``dwarf_gemm_bf16`` epilogue 3) ->
    ``dwarf_dsqg_fwd`` (resident-K/V kernel) with the ``if_gain`` and
    ``sigmoid(content_gate)`` epilogue fused -> out_proj GEMM. Otherwise: qkvg
    GEMM (tcgen05) -> ``dwarf_dsqg_prep`` -> ``dwarf_dsqg_fwd`` -> out_proj (tcgen05).
    """

    def __init__(self, embedding_dim, num_heads, offsets, j_small, j_large, seq_len=2048, dropout=0.1,
                 k_group_size=3, grouped_mode="baseline", verify_mode=False, max_group_size=None,
                 max_group_spread=None, plane_shift=0, pos_bias_scale=None, movt_dynamic_rms_target=None, *,
                 backend: str = "auto", train_phase_probes: bool = False, scale_embed_init_std: float = 0.01,
                 npci_strength_tau: float = 0.25, online_softmax: bool = True,
                 support_crop_projections: bool = True, support_crop_min_offset: int = 64,
                 kv_cache: str = "bf16"):
        super().__init__()
        dimension, heads = int(embedding_dim), int(num_heads)
        if dimension % heads:
            raise ValueError("embedding_dim must be divisible by num_heads")
        self.num_heads = heads
        self.head_dim = dimension // heads
        if self.head_dim < 16:
            raise ValueError("DSQG Triton paths require head_dim >= 16")
        self.seq_len = int(seq_len)
        self.backend = str(backend).lower()
        if self.backend not in {"auto", "eager", "triton"}:
            raise ValueError("backend must be auto, eager, or triton")
        if not math.isfinite(scale_embed_init_std) or scale_embed_init_std < 0:
            raise ValueError("scale_embed_init_std must be finite and non-negative")
        if not math.isfinite(npci_strength_tau) or npci_strength_tau <= 0:
            raise ValueError("npci_strength_tau must be finite and positive")
        if isinstance(support_crop_min_offset, bool) or int(support_crop_min_offset) < 0:
            raise ValueError("support_crop_min_offset must be a non-negative integer")
        if kv_cache not in ("bf16", "q6"):
            raise ValueError("kv_cache must be 'bf16' or 'q6'")
        self.kv_cache = kv_cache
        self.scale_embed_init_std = float(scale_embed_init_std)
        self.npci_strength_tau = float(npci_strength_tau)
        self.train_phase_probes = bool(train_phase_probes)
        self.support_crop_projections = bool(support_crop_projections)
        self.support_crop_min_offset = int(support_crop_min_offset)
        self.movt_dynamic_rms_target = None if movt_dynamic_rms_target is None else float(movt_dynamic_rms_target)
        self.movt_phase_gain_init_std = (
            0.001 if self.movt_dynamic_rms_target is None else calibrated_movt_phase_gain_std(
                head_dim=self.head_dim, target_dynamic_rms=self.movt_dynamic_rms_target, gate_logit=0.0)
        )
        self.grouped_mode = str(grouped_mode)
        self.grouped_mode_id = _resolve_grouped_mode(self.grouped_mode)
        self.online_softmax = bool(online_softmax) and self.grouped_mode == "baseline"
        self.verify_mode = bool(verify_mode)
        k_group_size, max_group_size, max_group_spread = _normalize_grouping_args(
            k_group_size, max_group_size, max_group_spread, self.grouped_mode_id
        )
        self.k_group_size, self.max_group_size, self.max_group_spread = k_group_size, max_group_size, max_group_spread
        self.plane_shift = _normalize_plane_shift(R_PLANES, self.head_dim, int(plane_shift))
        canonical, j_small, j_large = _canonicalize_offsets(list(offsets), j_small, j_large)
        self.offsets = tuple(canonical)
        self.j_val, self.j_small, self.j_large = len(canonical), int(j_small), int(j_large)
        if self.j_val < 1:
            raise ValueError("DSQG requires at least one offset")
        self.minimum_offset = min(self.offsets)
        self.register_buffer("offsets_dev", torch.tensor(canonical, dtype=torch.int32), persistent=False)
        plan = _plan_sparse_groups(canonical, self.j_small, k_group_size, max_group_size, max_group_spread)
        if self.verify_mode:
            _verify_sparse_plan(canonical, self.j_small, plan)
        for name in ("sparse_order", "group_start", "group_len", "group_dmin", "group_dmax"):
            self.register_buffer(f"{name}_dev", torch.tensor(plan[name], dtype=torch.int32), persistent=False)
        self.max_group_len = int(plan["max_group_len"])
        self.max_group_spread_observed = int(plan["max_group_spread"])
        self.num_sparse_groups = len(plan["group_len"])
        if pos_bias_scale is None:
            pos_bias_scale = _env_float("DWARF_DSQG_POS_BIAS_SCALE", 1.0)
        if not math.isfinite(float(pos_bias_scale)):
            raise ValueError("pos_bias_scale must be finite")
        self.register_buffer("pos_bias_scale", torch.tensor(float(pos_bias_scale), dtype=torch.float32),
                             persistent=True)

        self.qkvg_proj = nn.Linear(dimension, 4 * dimension, bias=True)
        self.out_proj = nn.Linear(dimension, dimension, bias=False)
        with torch.no_grad():
            self.qkvg_proj.bias.zero_()
        self.pos_bias_log_slope = nn.Parameter(torch.log(torch.expm1(torch.linspace(0.2, 2.0, heads))))
        self.pos_bias_residual = nn.Parameter(torch.zeros(self.j_val, heads))
        self.scale_embed = nn.Parameter(torch.randn(self.j_val, self.head_dim) * self.scale_embed_init_std)
        with torch.no_grad():
            self.scale_embed.sub_(self.scale_embed.mean(0, keepdim=True))
        self.if_gain = nn.Parameter(torch.ones(heads))
        self.phase_base = nn.Parameter(torch.randn(max(self.j_large, 1), heads, R_PLANES) * 0.01)
        self.phase_gain = nn.Parameter(
            torch.randn(max(self.j_large, 1), heads, R_PLANES) * self.movt_phase_gain_init_std
        )
        self.phase_gate = nn.Parameter(torch.zeros(max(self.j_large, 1)))
        qp, kp = _orthogonal_phase_probes(R_PLANES, self.head_dim, self.plane_shift)
        self.query_probes = nn.Parameter(qp, requires_grad=self.train_phase_probes)
        self.key_probes = nn.Parameter(kp, requires_grad=self.train_phase_probes)
        raw_theta = _raw_npci_theta_from_effective(NPCI_THETA_INIT)
        self.npci_theta_k = nn.Parameter(torch.full((heads,), raw_theta))
        self.npci_theta_v = nn.Parameter(torch.full((heads,), raw_theta))
        self.dropout = nn.Dropout(float(dropout))
        self._tables_cache: tuple | None = None

    # -- parameter-derived tables (reference :2981-2995, 3246-3256)
    @property
    def pos_bias(self) -> torch.Tensor:
        log_distance = torch.log1p(
            self.offsets_dev.to(device=self.pos_bias_residual.device, dtype=self.pos_bias_residual.dtype)
        ).reshape(-1, 1)
        slope = F.softplus(self.pos_bias_log_slope).reshape(1, -1)
        return (-log_distance * slope + self.pos_bias_residual) * self.pos_bias_scale

    @property
    def centered_scale_embed(self) -> torch.Tensor:
        return self.scale_embed - self.scale_embed.mean(dim=0, keepdim=True)

    def _migrate_legacy_keys(self, state_dict, prefix: str) -> None:
        """Rewrites, in place, the reference's older checkpoint layouts (dsqg_attention_v22.py:3069-3142).

        * separate ``qkv_proj`` / ``gate_proj`` weights and biases -> one ``qkvg_proj``
          (a missing gate keeps this module's current gate rows, missing biases are zero);
        * ``out_proj.bias`` is dropped (the projection is bias-free);
        * the old free ``pos_bias`` [J, H] table -> ``pos_bias_residual`` against this
          module's analytic slope, so the effective bias (analytic + residual) is unchanged;
        * absent ``pos_bias_*`` entries keep this module's current values.
        """
        D = self.qkvg_proj.in_features
        state_dict.pop(prefix + "out_proj.bias", None)
        w_key, b_key = prefix + "qkvg_proj.weight", prefix + "qkvg_proj.bias"
        if w_key not in state_dict and prefix + "qkv_proj.weight" in state_dict:
            qkv_w = state_dict.pop(prefix + "qkv_proj.weight")
            gate_w = state_dict.pop(prefix + "gate_proj.weight", None)
            if gate_w is None:
                gate_w = self.qkvg_proj.weight.detach()[3 * D:].clone()
            qkv_b = state_dict.pop(prefix + "qkv_proj.bias", None)
            if qkv_b is None:
                qkv_b = qkv_w.new_zeros(3 * D)
            gate_b = state_dict.pop(prefix + "gate_proj.bias", None)
            if gate_b is None:
                gate_b = qkv_b.new_zeros(D)
            state_dict[w_key] = torch.cat((qkv_w, gate_w), dim=0)
            state_dict[b_key] = torch.cat((qkv_b, gate_b), dim=0)
        old_key, res_key, slope_key = prefix + "pos_bias", prefix + "pos_bias_residual", prefix + "pos_bias_log_slope"
        if old_key in state_dict and res_key not in state_dict:
            old = state_dict.pop(old_key)
            slope = self.pos_bias_log_slope.detach().clone()
            state_dict[slope_key] = slope
            log_distance = torch.log1p(self.offsets_dev.to(device=old.device, dtype=old.dtype)).reshape(-1, 1)
            analytic = -log_distance * F.softplus(slope.to(device=old.device, dtype=old.dtype)).reshape(1, -1)
            state_dict[res_key] = old - analytic
        current = self.state_dict()
        for name in ("pos_bias_log_slope", "pos_bias_residual", "pos_bias_scale"):
            if prefix + name not in state_dict:
                state_dict[prefix + name] = current[name].detach().clone()

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                              error_msgs):
        self._migrate_legacy_keys(state_dict, prefix)
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                                      error_msgs)

    def _tables(self):
        """fp32 device tables the kernels read, recomputed only when a parameter changed."""
        params = (self.pos_bias_log_slope, self.pos_bias_residual, self.pos_bias_scale, self.scale_embed,
                  self.phase_base, self.phase_gain, self.phase_gate, self.query_probes, self.key_probes)
        key = tuple((p.data_ptr(), p._version) for p in params)
        if self._tables_cache is not None and self._tables_cache[0] == key:
            return self._tables_cache[1]
        with torch.no_grad():
            gate = torch.sigmoid(self.phase_gate.float())[:, None, None]
            tables = {
                "pos_bias": self.pos_bias.float().contiguous(),
                "scale_embed": self.centered_scale_embed.float().contiguous(),
                "phase_base": (self.phase_base.float() * gate).contiguous(),
                "phase_gain": (self.phase_gain.float() * gate).contiguous(),
                "q_probe": F.normalize(self.query_probes.float(), dim=-1).contiguous(),
                "k_probe": F.normalize(self.key_probes.float(), dim=-1).contiguous(),
                "offsets": self.offsets_dev.to(torch.int32).contiguous(),
            }
        self._tables_cache = (key, tables)
        return tables

    def reset_phase_probes_(self) -> None:
        q, k = _orthogonal_phase_probes(R_PLANES, self.head_dim, self.plane_shift)
        with torch.no_grad():
            self.query_probes.copy_(q.to(self.query_probes))
            self.key_probes.copy_(k.to(self.key_probes))

    def phase_probe_regularizer(self) -> torch.Tensor:
        if not self.train_phase_probes:
            return self.query_probes.sum() * 0.0
        q = F.normalize(self.query_probes.float(), dim=-1)
        k = F.normalize(self.key_probes.float(), dim=-1)
        eye = torch.eye(R_PLANES, device=q.device)
        return ((q @ q.t() - eye).square().mean() + (k @ k.t() - eye).square().mean()
                + (q @ k.t()).square().mean())

    def support_statistics(self, model_length: int | None = None) -> dict[str, object]:
        length = int(model_length if model_length is not None else self.seq_len - 1)
        support = [max(0, length - d) for d in self.offsets]
        return {
            "model_length": length,
            "offsets": self.offsets,
            "minimum_support": min(support),
            "maximum_support": max(support),
            "mean_valid_fraction": sum(support) / max(1, length * len(self.offsets)),
            "dead_offsets": tuple(d for d, s in zip(self.offsets, support, strict=True) if s == 0),
        }

    def semantic_config(self) -> dict[str, object]:
        return {
            "implementation": "dsqg-v22-fused",
            "offsets": self.offsets,
            "j_small": self.j_small,
            "j_large": self.j_large,
            "plane_shift": self.plane_shift,
            "positional_bias": "analytic_log_plus_residual",
            "pos_bias_scale": float(self.pos_bias_scale.detach().cpu()),
            "scale_embed": "centered_virtual_key",
            "phase_probes_trainable": self.train_phase_probes,
            "npci": "magnitude_aware",
            "npci_strength_tau": self.npci_strength_tau,
        }

    def execution_config(self) -> dict[str, object]:
        return {
            "backend": self.backend,
            "grouped_mode": self.grouped_mode,
            "online_softmax": self.online_softmax,
            "query_support_start": self.minimum_offset,
            "support_crop_projections": self.support_crop_projections,
            "support_crop_min_offset": self.support_crop_min_offset,
            "phase_probe_kernel": "dwarf_dsqg_prep",
            "k_group_size": self.k_group_size,
            "max_group_size": self.max_group_size,
            "max_group_spread": self.max_group_spread,
            "kv_cache": self.kv_cache,
        }

    def forward(self, x: torch.Tensor, kv_inject: tuple[torch.Tensor, torch.Tensor] | None = None) -> torch.Tensor:
        if self.backend == "eager":
            raise NotImplementedError("the B200 engine has no eager backend; construct with backend='auto'")
        _lib.require_cuda(x)
        if _needs_grad(x, *self.parameters()) or (self.training and self.dropout.p > 0):
            return self._forward_autograd(x, kv_inject)
        batch, seq_len, dimension = x.shape
        heads, head_dim = self.num_heads, self.head_dim
        query_start = min(self.minimum_offset, seq_len)
        key_end = max(0, seq_len - query_start)
        if query_start >= seq_len:
            return torch.zeros_like(x)
        act = torch.bfloat16
        xb = x if x.dtype == act else x.to(act)
        weight, bias = self.qkvg_proj.weight, self.qkvg_proj.bias
        t = self._tables()
        if kv_inject is None and self.kv_cache == "q6" and head_dim == 64 and dimension % 256 == 0:
            # qkvg GEMM on tcgen05 with the prep pass (probes, q6 pack) in its epilogue.
            qkvg, y_pre, z_pre, cache = gemm.qkvg_prep(xb, weight.to(act), bias.to(act), heads, t["q_probe"],
                                                       t["k_probe"])
            query = qkvg.view(batch, seq_len, 4, heads, head_dim)[:, :, 0].permute(0, 2, 1, 3)
            return self._attend(x, query, ("q6", *cache), y_pre, z_pre, qkvg[:, :, 3 * dimension:], t,
                                query_start)
        qkvg = gemm.linear(xb, weight.to(act), bias.to(act))  # [B, N, 4D]
        split = qkvg.view(batch, seq_len, 4, heads, head_dim)
        query = split[:, :, 0].permute(0, 2, 1, 3)
        key = split[:, :, 1].permute(0, 2, 1, 3)
        value = split[:, :, 2].permute(0, 2, 1, 3)
        content_gate = qkvg[:, :, 3 * dimension:]
        if kv_inject is not None:
            key_delta, value_delta = kv_inject
            full = key.shape
            prefix = (batch, heads, key_end, head_dim)
            if key_delta.shape == full and value_delta.shape == full:
                kd, vd = key_delta[:, :, :key_end], value_delta[:, :, :key_end]
            elif key_delta.shape == prefix and value_delta.shape == prefix:
                kd, vd = key_delta, value_delta
            else:
                raise ValueError(
                    "kv_inject must contain full [B,H,N,HD] tensors or the "
                    "exact live source prefix [B,H,N-min_offset,HD]"
                )
            rk = npci_rotate(key[:, :, :key_end], kd, NPCI_THETA_MAX * torch.tanh(self.npci_theta_k),
                             strength_tau=self.npci_strength_tau)
            rv = npci_rotate(value[:, :, :key_end], vd, NPCI_THETA_MAX * torch.tanh(self.npci_theta_v),
                             strength_tau=self.npci_strength_tau)
            key = torch.cat((rk, key[:, :, key_end:]), dim=2) if key_end < seq_len else rk
            value = torch.cat((rv, value[:, :, key_end:]), dim=2) if key_end < seq_len else rv
        q6 = self.kv_cache == "q6"
        y_pre, z_pre, cache = dsqg_prep(query, key, value, t["q_probe"], t["k_probe"], pack_q6=q6)
        kv = ("q6", *cache) if q6 else ("bf16", key, value)
        return self._attend(x, query, kv, y_pre, z_pre, content_gate, t, query_start)

    def _forward_autograd(self, x: torch.Tensor, kv_inject=None) -> torch.Tensor:
        """Differentiable forward (training): the reference forward (:3144-3289,
        without the support-crop projection schedule, which computes the same
        values) with the projections, probes and tables as torch ops and the
        attention on ``dwarf_dsqg_fwd`` / ``dwarf_dsqg_bwd`` (bf16 K/V)."""
        batch, seq_len, dimension = x.shape
        heads, head_dim = self.num_heads, self.head_dim
        query_start = min(self.minimum_offset, seq_len)
        key_end = max(0, seq_len - query_start)
        if query_start >= seq_len:
            return torch.zeros_like(x)
        q_flat, k_flat, v_flat, content_gate = self.qkvg_proj(x).split(dimension, dim=-1)
        query = q_flat.reshape(batch, seq_len, heads, head_dim).permute(0, 2, 1, 3)
        key = k_flat.reshape(batch, seq_len, heads, head_dim).permute(0, 2, 1, 3)
        value = v_flat.reshape(batch, seq_len, heads, head_dim).permute(0, 2, 1, 3)
        if kv_inject is not None:
            key_delta, value_delta = kv_inject
            full = key.shape
            prefix = (batch, heads, key_end, head_dim)
            if key_delta.shape == full and value_delta.shape == full:
                kd, vd = key_delta[:, :, :key_end], value_delta[:, :, :key_end]
            elif key_delta.shape == prefix and value_delta.shape == prefix:
                kd, vd = key_delta, value_delta
            else:
                raise ValueError(
                    "kv_inject must contain full [B,H,N,HD] tensors or the "
                    "exact live source prefix [B,H,N-min_offset,HD]"
                )
            rk = npci_rotate_autograd(key[:, :, :key_end], kd, NPCI_THETA_MAX * torch.tanh(self.npci_theta_k),
                                      strength_tau=self.npci_strength_tau)
            rv = npci_rotate_autograd(value[:, :, :key_end], vd, NPCI_THETA_MAX * torch.tanh(self.npci_theta_v),
                                      strength_tau=self.npci_strength_tau)
            key = torch.cat((rk, key[:, :, key_end:]), dim=2) if key_end < seq_len else rk
            value = torch.cat((rv, value[:, :, key_end:]), dim=2) if key_end < seq_len else rv
        query_probe = F.normalize(self.query_probes.float(), dim=-1)
        key_probe = F.normalize(self.key_probes.float(), dim=-1)
        qf, kf = query.float(), key.float()
        eps = 1e-6 * head_dim
        y_pre = (torch.einsum("bhnd,rd->bhnr", qf, query_probe)
                 * torch.rsqrt(qf.square().sum(-1, keepdim=True) + eps)).contiguous()
        z_pre = (torch.einsum("bhnd,rd->bhnr", kf, key_probe)
                 * torch.rsqrt(kf.square().sum(-1, keepdim=True) + eps)).contiguous()
        phase_gate = torch.sigmoid(self.phase_gate)[:, None, None]
        output = dsqg_attention_v18_grouped(
            query, key, value, self.pos_bias, self.centered_scale_embed, self.phase_base * phase_gate,
            self.phase_gain * phase_gate, y_pre, z_pre, self.j_val, self.j_small, self.j_large, self.offsets_dev,
            None, None, None, None, None, self.k_group_size, 0, False, 0, self.plane_shift, query_start)
        output = output.to(x.dtype) * self.if_gain.reshape(1, heads, 1, 1).to(x.dtype)
        flattened = output.permute(0, 2, 1, 3).reshape(batch, seq_len, dimension)
        return self.dropout(self.out_proj(flattened * torch.sigmoid(content_gate)))

    def forward_cached(self, x: torch.Tensor, cache, row: int) -> torch.Tensor:
        """Attention output for positions [row, row + T) of ``x`` [B,T,D], appending their
        q6 K/V (and the K-side phase probes) to ``cache`` first.

        ``cache`` = (y, z, k_codes, k_scales, v_codes, v_scales) of L positions per
        (batch, head) (the layout ``gemm.qkvg_prep`` documents) holding positions
        [0, row). row = 0 is a prefill; T = 1 is one decode step, whose DSQG launch
        computes the single query row over the whole cache.
        """
        _lib.require_cuda(x)
        if torch.is_grad_enabled():
            _forward_only(x, *self.parameters())
        if self.kv_cache != "q6" or self.head_dim != 64 or (self.num_heads * 64) % 256 != 0:
            raise NotImplementedError("cached (incremental) DSQG runs on the q6 cache with head_dim 64")
        batch, rows, dimension = x.shape
        heads, head_dim = self.num_heads, self.head_dim
        act = torch.bfloat16
        xb = x if x.dtype == act else x.to(act)
        t = self._tables()
        qkvg, y_pre, _, _ = gemm.qkvg_prep(xb, self.qkvg_proj.weight.to(act), self.qkvg_proj.bias.to(act), heads,
                                           t["q_probe"], t["k_probe"], cache=cache, row=row)
        seq_len = row + rows
        query_start = min(self.minimum_offset, seq_len)
        if query_start >= seq_len:
            return torch.zeros_like(x)
        query = qkvg.view(batch, rows, 4, heads, head_dim)[:, :, 0].permute(0, 2, 1, 3)
        _, z, kc, ks, vc, vs = cache
        return self._attend(x, query, ("q6", kc, ks, vc, vs), y_pre, z, qkvg[:, :, 3 * dimension:], t,
                            query_start, seq_len=seq_len, row_begin=row)

    def forward_step(self, x: torch.Tensor, cache, pos: torch.Tensor) -> torch.Tensor:
        """One new token per sequence (x [B,1,D]) at the device position ``pos`` (int64 [1]):
        the q6 append and the DSQG launch both read the position from device memory, so
        the step can be captured once in a CUDA graph and replayed at every position."""
        if self.kv_cache != "q6" or self.head_dim != 64 or (self.num_heads * 64) % 256 != 0:
            raise NotImplementedError("cached (incremental) DSQG runs on the q6 cache with head_dim 64")
        batch, rows, dimension = x.shape
        if rows != 1:
            raise ValueError("forward_step takes one token per sequence")
        heads, head_dim = self.num_heads, self.head_dim
        act = torch.bfloat16
        xb = x if x.dtype == act else x.to(act)
        t = self._tables()
        qkvg, _, _, _ = gemm.qkvg_prep(xb, self.qkvg_proj.weight.to(act), self.qkvg_proj.bias.to(act), heads,
                                       t["q_probe"], t["k_probe"], cache=cache, pos=pos)
        query = qkvg.view(batch, 1, 4, heads, head_dim)[:, :, 0].permute(0, 2, 1, 3)
        y, z, kc, ks, vc, vs = cache
        return self._attend(x, query, ("q6", kc, ks, vc, vs), y, z, qkvg[:, :, 3 * dimension:], t,
                            self.minimum_offset, seq_len=1, pos=pos)

    def _attend(self, x, query, kv, y_pre, z_pre, content_gate, t, query_start, *, seq_len=None, row_begin=0,
                pos=None):
        """DSQG kernel (if_gain and content-gate epilogue fused) followed by out_proj.

        With ``row_begin`` > 0 ``query``/``y_pre``/``content_gate`` hold positions
        [row_begin, seq_len) and K/V, z_pre positions [0, seq_len)."""
        act = torch.bfloat16
        batch, heads, rows, head_dim = query.shape
        dimension = heads * head_dim
        out = torch.empty(batch, rows, dimension, dtype=act, device=x.device)
        out_view = out.view(batch, rows, heads, head_dim).permute(0, 2, 1, 3)
        gain = self.if_gain if self.if_gain.dtype in (torch.bfloat16, torch.float32) else self.if_gain.float()
        _dsqg_launch(query, kv=kv, pos_bias=t["pos_bias"], scale_embed=t["scale_embed"],
                     phase_base=t["phase_base"], phase_gain=t["phase_gain"], y_pre=y_pre, z_pre=z_pre,
                     offsets=t["offsets"], j_small=self.j_small, j_large=self.j_large,
                     plane_shift=self.plane_shift, query_start=query_start, out=out_view,
                     head_gain=gain.detach().contiguous(), gate=content_gate, seq_len=seq_len,
                     row_begin=row_begin, pos=pos)
        result = gemm.linear(out, self.out_proj.weight.to(act))
        return self.dropout(result).to(x.dtype) if x.dtype != act else self.dropout(result)


DSQGAttentionV20 = DSQGAttentionV19
DSQGAttentionV21 = DSQGAttentionV19
DSQGAttentionV22 = DSQGAttentionV19
