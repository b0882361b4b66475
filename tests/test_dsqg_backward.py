"""DSQG backward: the oracle's gradients (fp64 autograd through
oracle.dsqg.dsqg_forward_torch) pinned to golden vectors made by fp64 autograd
through the reference's ``_eager_dsqg_attention`` (CPU), and the engine's
autograd path (``dwarf_dsqg_fwd`` + ``dwarf_dsqg_bwd`` through the C ABI)
checked against the oracle (GPU).

Tolerances: the north-star bf16 attention bar, 2e-2 max-abs and 1e-2 mean
relative error, applied to each gradient after scaling by its largest
magnitude (gradients such as d pos_bias sum thousands of terms).
"""

import numpy as np
import pytest
import torch

from oracle import dsqg as oracle_dsqg
from tests._golden import load

NAMES = ("q", "k", "v", "pos_bias", "scale_embed", "phase_base", "phase_gain", "y_pre", "z_pre")
CASES = [("dsqg_config1", "dsqg_bwd_config1"), ("dsqg_gqa_ragged", "dsqg_bwd_gqa_ragged")]


def _offsets(g):
    return [int(o) for o in g["offsets"]]


@pytest.mark.parametrize("src,dst", CASES)
def test_oracle_backward_matches_reference_autograd(src, dst):
    g, gb = load(src), load(dst)
    grads = oracle_dsqg.dsqg_backward({n: g[n] for n in NAMES}, gb["dout"], _offsets(g), int(g["j_small"]),
                                      int(g["plane_shift"]), 0, round_scale_embed=False)
    for n in NAMES:
        ref = gb["d_" + n].double()
        assert (grads["d_" + n] - ref).abs().max() <= 1e-5 * max(1.0, float(ref.abs().max())), n


def _assert_grad_close(got: torch.Tensor, ref: torch.Tensor, name: str):
    got, ref = got.detach().double().cpu(), ref.double()
    scale = max(1.0, float(ref.abs().max()))
    err = (got - ref).abs()
    assert float(err.max()) <= 2e-2 * scale, f"{name}: max-abs {float(err.max()):.3g} (scale {scale:.3g})"
    mean_rel = float(err.mean()) / max(float(ref.abs().mean()), 1e-12)
    assert mean_rel <= 1e-2, f"{name}: mean-rel {mean_rel:.3g}"


def _engine_grads(inputs: dict, dout, offsets, j_small, j_large, plane_shift, query_start):
    from dwarf_v2_b200.dsqg_attention_v22 import dsqg_attention_v18_grouped

    leaves = {n: inputs[n].cuda().requires_grad_(True) for n in NAMES}
    offs = torch.tensor(offsets, dtype=torch.int32, device="cuda")
    empty = torch.empty(0, dtype=torch.int32, device="cuda")
    out = dsqg_attention_v18_grouped(*(leaves[n] for n in NAMES), j_small + j_large, j_small, j_large, offs,
                                     empty, empty, empty, empty, empty, 3, 0, False, 0, plane_shift, query_start)
    out.backward(dout.cuda())
    torch.cuda.synchronize()
    return out, {"d_" + n: leaves[n].grad for n in NAMES}


@pytest.mark.gpu
@pytest.mark.parametrize("src,dst", CASES)
def test_engine_backward_matches_oracle(src, dst):
    g, gb = load(src), load(dst)
    js, jl = int(g["j_small"]), int(g["j_large"])
    ps, qs = int(g["plane_shift"]), int(g["query_start"])
    inputs = {n: g[n] if n in ("q", "k", "v") else g[n].float() for n in NAMES}
    _, grads = _engine_grads(inputs, gb["dout"], _offsets(g), js, jl, ps, qs)
    ref = oracle_dsqg.dsqg_backward({n: g[n] for n in NAMES}, gb["dout"], _offsets(g), js, ps, qs)
    for n in NAMES:
        _assert_grad_close(grads["d_" + n], ref["d_" + n], n)
    assert grads["d_q"].dtype == torch.bfloat16 and grads["d_pos_bias"].dtype == torch.float32


def _model_group_case(seed: int, B: int, H: int, H_kv: int, N: int):
    """The model's first DSQG offset group (29 offsets: 6 small, 23 large) with
    random tables of the magnitudes the fixtures use."""
    all_offsets = [1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 13, 15, 16, 19, 21, 23, 28, 48, 64, 96, 121, 161, 192, 212, 245,
                   273, 295, 342, 375, 384, 413, 441, 473, 512, 549, 579, 593, 631, 653, 694, 716, 768, 826, 846,
                   900, 936, 970, 1000, 1024, 1074, 1108, 1144, 1166, 1190, 1218, 1244, 1288, 1322, 1385, 1423,
                   1451, 1497, 1522, 1550, 1581, 1603, 1617, 1634, 1651, 1661, 1710, 1743, 1780, 1810, 1820,
                   1852, 1860, 1876, 1886, 1897, 1903, 1916, 1926, 1929, 1941, 1965, 1983, 2006, 2011, 2029,
                   2037, 2044]
    offsets = [o for o in all_offsets if 2048 - o >= 64][0::3]
    js = sum(1 for o in offsets if o <= 28)
    J = len(offsets)
    gen = torch.Generator().manual_seed(seed)
    r = lambda *s, std=1.0: torch.randn(*s, generator=gen) * std  # noqa: E731
    inputs = dict(q=r(B, H, N, 64).bfloat16(), k=r(B, H_kv, N, 64).bfloat16(), v=r(B, H_kv, N, 64).bfloat16(),
                  pos_bias=r(J, H, std=0.3), scale_embed=r(J, 64, std=0.3), phase_base=r(J - js, H, 4, std=0.7),
                  phase_gain=r(J - js, H, 4, std=2.0), y_pre=r(B, H, N, 4, std=0.5).clamp(-1, 1),
                  z_pre=r(B, H_kv, N, 4, std=0.5).clamp(-1, 1))
    dout = r(B, H, N, 64).bfloat16()
    return inputs, dout, offsets, js, J - js


@pytest.mark.gpu
def test_engine_backward_model_group_full_length():
    """T=2048 with the model's 29-offset group (the training shape of one DSQG layer, one row)."""
    inputs, dout, offsets, js, jl = _model_group_case(7, 1, 8, 8, 2048)
    _, grads = _engine_grads(inputs, dout, offsets, js, jl, 0, 0)
    ref = oracle_dsqg.dsqg_backward(inputs, dout, offsets, js, 0, 0)
    for n in NAMES:
        _assert_grad_close(grads["d_" + n], ref["d_" + n], n)


@pytest.mark.gpu
def test_engine_backward_properties_batch():
    """B=8 rows: the gradients of each batch row equal those of the row run alone
    (rows are independent), and two runs give identical dq/dk/dv (no atomics there)."""
    inputs, dout, offsets, js, jl = _model_group_case(8, 8, 8, 8, 512)
    out, grads = _engine_grads(inputs, dout, offsets, js, jl, 0, 0)
    _, grads2 = _engine_grads(inputs, dout, offsets, js, jl, 0, 0)
    for n in ("d_q", "d_k", "d_v", "d_y_pre", "d_z_pre"):
        assert torch.equal(grads[n], grads2[n]), n
    row = {n: (t[3:4] if n in ("q", "k", "v", "y_pre", "z_pre") else t) for n, t in inputs.items()}
    _, g1 = _engine_grads(row, dout[3:4], offsets, js, jl, 0, 0)
    for n in ("d_q", "d_k", "d_v", "d_y_pre", "d_z_pre"):
        assert torch.equal(grads[n][3:4], g1[n]), n


@pytest.mark.gpu
@pytest.mark.parametrize("tag", ["plain", "inject"])
def test_module_training_gradients_match_reference(tag):
    """DSQGAttentionV19 in training mode (fp32 parameters, bf16 attention on the
    engine) against the reference module's CPU fp32 gradients: dx and every
    parameter gradient, with and without a kv_inject packet."""
    from dwarf_v2_b200.dsqg_attention_v22 import DSQGAttentionV19

    g = load("dsqg_module_grad")
    module = DSQGAttentionV19(128, 2, [1, 2, 3, 5, 8, 13, 21, 48, 64, 100], 7, 3, seq_len=160, dropout=0.0,
                              plane_shift=6).train()
    module.load_state_dict({k[len("state."):]: v for k, v in g.items() if k.startswith("state.")})
    module = module.cuda()
    x = g["x"].cuda().requires_grad_(True)
    inject = (g["kd"].cuda(), g["vd"].cuda()) if tag == "inject" else None
    y = module(x, inject)
    y.backward(g["dy"].cuda())
    _assert_grad_close(y, g[f"{tag}.y"], "y")
    _assert_grad_close(x.grad, g[f"{tag}.dx"], "dx")
    prefix = f"{tag}.grad."
    names = [k[len(prefix):] for k in g if k.startswith(prefix)]
    assert "qkvg_proj.weight" in names and "pos_bias_residual" in names
    params = dict(module.named_parameters())
    for name in names:
        assert params[name].grad is not None, name
        _assert_grad_close(params[name].grad, g[prefix + name], name)
