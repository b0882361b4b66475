"""HISA fused tile attention backward: the oracle's gradients (fp64 autograd through
oracle.hisa.attention_torch) pinned to golden vectors made by fp64 autograd through
the reference's own eager lanes + LSE merge (CPU), and the engine's autograd path
(``dwarf_hisa_attn`` + ``dwarf_hisa_attn_bwd`` through the C ABI) checked against
the oracle (GPU).

Tolerances: the north-star bf16 attention bar, 2e-2 max-abs and 1e-2 mean relative
error, applied to each gradient after scaling by its largest magnitude.
"""

import pytest
import torch

from oracle import hisa as oracle_hisa
from tests._golden import load

NAMES = ("query", "local_key", "local_value", "global_key", "global_value", "route")
FIXTURE_KEYS = dict(query="q", local_key="local_key", local_value="local_value", global_key="global_key",
                    global_value="global_value", route="route")


def _inputs(g):
    return {n: g[FIXTURE_KEYS[n]] for n in NAMES}


def test_oracle_backward_matches_reference_autograd():
    g, gb = load("hisa_router_lanes"), load("hisa_bwd_lanes")
    grads = oracle_hisa.attention_backward(_inputs(g), gb["dout"], g["top_chunk_idx"], g["valid_lengths"])
    for n in NAMES:
        ref = gb["d_" + FIXTURE_KEYS[n]].double()
        assert (grads["d_" + n] - ref).abs().max() <= 1e-5 * max(1.0, float(ref.abs().max())), n


def _assert_grad_close(got, ref, name):
    got, ref = got.detach().double().cpu(), ref.double()
    scale = max(1.0, float(ref.abs().max()))
    err = (got - ref).abs()
    assert float(err.max()) <= 2e-2 * scale, f"{name}: max-abs {float(err.max()):.3g} (scale {scale:.3g})"
    mean_rel = float(err.mean()) / max(float(ref.abs().mean()), 1e-12)
    assert mean_rel <= 1e-2, f"{name}: mean-rel {mean_rel:.3g}"


def _engine(inputs, dout, top, lengths):
    from dwarf_v2_b200.hierarchical_sparse_attn_v18_hisa import hisa_tile_attention

    leaves = {n: inputs[n].cuda().requires_grad_(True) for n in NAMES}
    out = hisa_tile_attention(*(leaves[n] for n in NAMES), top.cuda(), lengths.cuda())
    out.backward(dout.cuda())
    torch.cuda.synchronize()
    return out, {"d_" + n: leaves[n].grad for n in NAMES}


@pytest.mark.gpu
def test_engine_backward_matches_reference_golden():
    """Ragged T=300 (5 chunks, the last partial), per-row valid lengths 300 / 250."""
    g, gb = load("hisa_router_lanes"), load("hisa_bwd_lanes")
    out, grads = _engine(_inputs(g), gb["dout"], g["top_chunk_idx"], g["valid_lengths"])
    _assert_grad_close(out, g["merged"], "out")
    ref = oracle_hisa.attention_backward(_inputs(g), gb["dout"], g["top_chunk_idx"], g["valid_lengths"])
    for n in NAMES:
        _assert_grad_close(grads["d_" + n], ref["d_" + n], n)
        _assert_grad_close(grads["d_" + n], gb["d_" + FIXTURE_KEYS[n]], n + " (reference)")


@pytest.mark.gpu
def test_engine_backward_full_length():
    """T=2048 with the reference router's top-4 of up to 31 completed chunks."""
    g = load("hisa_router_long")
    gen = torch.Generator().manual_seed(61)
    B, H, T, D = g["q"].shape
    inputs = dict(query=g["q"], global_key=g["global_key"], route=g["route"],
                  local_key=(torch.randn(B, H, T, D, generator=gen) * 0.125).bfloat16(),
                  local_value=torch.randn(B, H, T, D, generator=gen).bfloat16(),
                  global_value=torch.randn(B, H, T, D, generator=gen).bfloat16())
    dout = torch.randn(B, H, T, D, generator=gen).bfloat16()
    _, grads = _engine(inputs, dout, g["top_chunk_idx"], g["valid_lengths"])
    ref = oracle_hisa.attention_backward(inputs, dout, g["top_chunk_idx"], g["valid_lengths"])
    for n in NAMES:
        _assert_grad_close(grads["d_" + n], ref["d_" + n], n)
    # every gradient row has one writer: runs are reproducible bit for bit
    _, again = _engine(inputs, dout, g["top_chunk_idx"], g["valid_lengths"])
    for n in NAMES:
        assert torch.equal(grads["d_" + n], again["d_" + n]), n


EDGE_CASES = ("t64", "t1", "t83", "t200")
EDGE_FIELDS = dict(query="q", local_key="local_key", local_value="local_value", global_key="global_key",
                   global_value="global_value", route="route")


def _edge(g, tag):
    return {n: g[f"{tag}.{f}"] for n, f in EDGE_FIELDS.items()}


@pytest.mark.parametrize("tag", EDGE_CASES)
def test_oracle_backward_edges_match_reference_autograd(tag):
    """T=64 (no routed chunk anywhere), T=1 (row 0 has no key), T=83 with a row of
    valid length 0 and a partial last tile, T=200 with lengths 130 / 199: the
    oracle's gradients against fp64 autograd through the reference's own router,
    lanes and merge."""
    g = load("hisa_bwd_edges")
    grads = oracle_hisa.attention_backward(_edge(g, tag), g[f"{tag}.dout"], g[f"{tag}.top_chunk_idx"],
                                           g[f"{tag}.valid_lengths"])
    for n, f in EDGE_FIELDS.items():
        ref = g[f"{tag}.d_{f}"].double()
        assert (grads["d_" + n] - ref).abs().max() <= 1e-5 * max(1.0, float(ref.abs().max())), n


@pytest.mark.gpu
@pytest.mark.parametrize("tag", EDGE_CASES)
def test_engine_backward_edges(tag):
    """The engine on the edge cases: route priors with fewer than 4 slots are padded
    with zero slots (the engine's route layout is [B,H,T,4]); rows past a valid
    length, and the whole length-0 row, get exactly zero gradients."""
    g = load("hisa_bwd_edges")
    inputs = _edge(g, tag)
    K = inputs["route"].shape[-1]
    padded = dict(inputs, route=torch.nn.functional.pad(inputs["route"], (0, 4 - K)))
    out, grads = _engine(padded, g[f"{tag}.dout"], g[f"{tag}.top_chunk_idx"], g[f"{tag}.valid_lengths"])
    _assert_grad_close(out, g[f"{tag}.merged"], "out")
    grads["d_route"] = grads["d_route"][..., :K]
    assert all(bool(torch.isfinite(v).all()) for v in grads.values())
    for n, f in EDGE_FIELDS.items():
        _assert_grad_close(grads["d_" + n], g[f"{tag}.d_{f}"], n)
    lengths = g[f"{tag}.valid_lengths"]
    for b in range(lengths.numel()):
        L = int(lengths[b])
        assert torch.all(grads["d_query"][b, :, L:] == 0) and torch.all(out[b, :, L:] == 0)
