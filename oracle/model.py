"""CPU oracle: whole DWARF-v2 prefill -- TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Restates ``DwarfForCausalLM.forward`` of train/train_dwarf.py:218-470 in
float32/float64 on the CPU, from a state dict with the reference's key
layout, composing the per-path oracles (oracle/dsqg.py, oracle/hisa.py,
oracle/ema.py) with torch CPU GEMMs:

* DSQG block (:299-322, kernels/dsqg_attention_v22.py:3144-3289): RMSNorm,
  qkvg projection, probe projections, DSQG attention, if_gain, content gate,
  out_proj, residual, SwiGLU FFN, residual;
* HISA block (:325-364, kernels/hierarchical_sparse_attn_v18_hisa.py:2546-2787):
  RMSNorm, EMA interference packet (:260-284), qkvg, low-rank global adapters,
  NPCI rotation (:99-125), router, joint local+routed attention, W_o and
  output gate, residual, FFN, residual;
* final RMSNorm and the tied lm_head.

Used as the parity anchor for the engine's model (pinned to the reference's
fp32 logits in tests/golden) and as the timed CPU baseline of bench.py.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from . import dsqg as odsqg
from . import ema as oema
from . import hisa as ohisa

LAYOUT = (0, 1, 2, None, 0, 1, 2, 0, 1, 2)


def _rms(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    return x * torch.rsqrt(x.square().mean(-1, keepdim=True) + eps) * w


def _ffn(x, sd, p):
    up, gate = torch.nn.functional.linear(x, sd[p + "ffn.up_gate.weight"]).chunk(2, dim=-1)
    return torch.nn.functional.linear(torch.nn.functional.silu(gate) * up, sd[p + "ffn.down.weight"])


def _heads(t: torch.Tensor, H: int) -> np.ndarray:
    B, T, D = t.shape
    return t.reshape(B, T, H, D // H).permute(0, 2, 1, 3).double().numpy()


def _npci(x: np.ndarray, d: np.ndarray, theta: np.ndarray, tau: float = 0.25) -> np.ndarray:
    norm = np.maximum(np.linalg.norm(x, axis=-1, keepdims=True), 1e-12)
    unit = x / norm
    perp = d - (d * unit).sum(-1, keepdims=True) * unit
    pn = np.linalg.norm(perp, axis=-1, keepdims=True)
    active = pn > norm * 1e-7
    direction = np.where(active, perp / np.maximum(pn, 1e-20), 0.0)
    angle = theta.reshape(1, -1, 1, 1) * np.tanh(pn / (tau * norm + 1e-12))
    return np.where(active, np.cos(angle) * x + np.sin(angle) * norm * direction, x)


def _dsqg_block(x, sd, p, offsets, j_small, plane_shift, H):
    B, T, D = x.shape
    n = _rms(x, sd[p + "norm1.weight"])
    a = p + "attn."
    q, k, v, gate = torch.nn.functional.linear(n, sd[a + "qkvg_proj.weight"], sd[a + "qkvg_proj.bias"]).split(D, -1)
    qh, kh, vh = _heads(q, H), _heads(k, H), _heads(v, H)
    y = odsqg.probe_projection(qh, sd[a + "query_probes"].double().numpy())
    z = odsqg.probe_projection(kh, sd[a + "key_probes"].double().numpy())
    pb, se, pbase, pgain = odsqg.derived_tables(
        offsets, sd[a + "pos_bias_log_slope"], sd[a + "pos_bias_residual"], float(sd[a + "pos_bias_scale"]),
        sd[a + "scale_embed"], sd[a + "phase_base"], sd[a + "phase_gain"], sd[a + "phase_gate"])
    out, _ = odsqg.dsqg_forward(qh, kh, vh, pb, se, pbase, pgain, y, z, offsets, j_small, plane_shift,
                                min(offsets), round_scale_embed=False)
    out = out * sd[a + "if_gain"].double().numpy().reshape(1, H, 1, 1)
    flat = torch.from_numpy(out).permute(0, 2, 1, 3).reshape(B, T, D).float()
    x = x + torch.nn.functional.linear(flat * torch.sigmoid(gate), sd[a + "out_proj.weight"])
    return x + _ffn(_rms(x, sd[p + "norm2.weight"]), sd, p)


def _hisa_block(x, sd, p, H):
    B, T, D = x.shape
    n = _rms(x, sd[p + "norm1.weight"])
    # EMA interference packet (train_dwarf.py:260-284)
    k = p + "packet."
    alphas = 1e-5 + (0.5 - 1e-5) * torch.sigmoid(sd[k + "ema_raw"]).double().numpy()
    scans = [oema.ema_scan(n.numpy(), a, clamp=(1e-5, 0.5)) for a in alphas]
    mix = torch.softmax(sd[k + "mix_logits"].double(), 0).numpy()
    pooled = sum(w * s for w, s in zip(mix, scans))
    ms = (pooled ** 2).mean(-1, keepdims=True)
    direction = pooled / np.sqrt(ms + 1e-6)
    gate_p = torch.sigmoid(torch.nn.functional.linear(n, sd[k + "gate_proj.weight"], sd[k + "gate_proj.bias"]))
    packet = torch.from_numpy(direction * np.tanh(np.sqrt(ms) / 0.25)).float() * gate_p
    kd, vd = torch.nn.functional.linear(packet, sd[k + "kv_proj.weight"]).chunk(2, -1)
    # projections, adapters, NPCI (hierarchical_sparse_attn_v18_hisa.py:2565-2605)
    a = p + "attn."
    q, kk, vv, gate = torch.nn.functional.linear(n, sd[a + "qkvg_proj.weight"], sd[a + "qkvg_proj.bias"]).split(D, -1)
    gk = kk + torch.nn.functional.linear(torch.nn.functional.linear(n, sd[a + "global_k_down.weight"]), sd[a + "global_k_up.weight"])
    gv = vv + torch.nn.functional.linear(torch.nn.functional.linear(n, sd[a + "global_v_down.weight"]), sd[a + "global_v_up.weight"])
    tk = 0.25 * np.tanh(sd[a + "npci_theta_k"].double().numpy())
    tv = 0.25 * np.tanh(sd[a + "npci_theta_v"].double().numpy())
    gkh = _npci(_heads(gk, H), _heads(kd, H), tk)
    gvh = _npci(_heads(gv, H), _heads(vd, H), tv)
    qh = _heads(q, H)
    lengths = np.full(B, T)
    reps = ohisa.chunk_representatives(gkh, lengths)
    top, _ = ohisa.select_chunks(qh, reps, lengths)
    scale = np.logaddexp(0.0, sd[a + "route_prior_raw"].double().numpy())
    route = ohisa.route_scores(qh, reps, top, scale)
    att = ohisa.attention(qh, _heads(kk, H), _heads(vv, H), gkh, gvh, route, top, lengths)
    merged = torch.from_numpy(att).permute(0, 2, 1, 3).reshape(B, T, D).float()
    x = x + torch.nn.functional.linear(merged, sd[a + "W_o.weight"]) * torch.sigmoid(gate)
    return x + _ffn(_rms(x, sd[p + "norm2.weight"]), sd, p)


def offset_groups(model_length: int = 2047, min_support: int = 64, all_offsets=None):
    live = [d for d in sorted(all_offsets) if model_length - d >= min_support]
    return [live[i::3] for i in range(3)]


@torch.no_grad()
def prefill(state_dict: dict, input_ids: torch.Tensor, *, all_offsets, heads: int = 8,
            return_hidden: bool = False) -> torch.Tensor:
    """fp32/fp64 CPU forward of the reference model; returns logits [B,T,V] (or final hidden)."""
    sd = {k: v.detach().float().cpu() for k, v in state_dict.items()}
    groups = offset_groups(all_offsets=all_offsets)
    x = sd["embedding.weight"][input_ids.cpu()]
    dsqg_index = 0
    for i, group in enumerate(LAYOUT):
        p = f"blocks.{i}."
        if group is None:
            x = _hisa_block(x, sd, p, heads)
            continue
        offs = groups[group]
        small = [d for d in offs if d <= 28]
        x = _dsqg_block(x, sd, p, sorted(small) + sorted(d for d in offs if d >= 48), len(small),
                        2 * (dsqg_index % 8), heads)
        dsqg_index += 1
    hidden = _rms(x, sd["norm.weight"])
    return hidden if return_hidden else torch.nn.functional.linear(hidden, sd["embedding.weight"])
