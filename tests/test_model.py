"""Whole-model drop-in: construction API and prefill parity with the reference.

CPU: DwarfForCausalLM builds the reference topology with bit-identical seeded
weights (parameter count and a SHA-256 over the state dict, captured from the
reference by tests/golden/make_golden.py). GPU: bf16 prefill of the reference
config (B=1, T=2048) against the reference's own forward.

Logit tolerance. The north-star 2e-2 max-abs logit tolerance is tighter than
the reference's own bf16 rounding noise on this random-init model: its bf16
run and its fp32 run differ by 0.045 max-abs / 2.1% mean-relative (the
fixture holds both). The bar used here is therefore "no worse than the
reference's own bf16 path": against the fp32 reference, the engine's logit
error may be at most 1.5x the reference bf16 run's error (max and mean), and
against the reference bf16 run at most 0.08 max-abs / 2.5% mean-relative.
The q6-KV model is compared with the reference run on q6-round-tripped K/V
(the q6 perturbation itself moves logits by 0.13 / 6%).
"""

import hashlib

import numpy as np
import pytest
import torch

from tests._golden import load


def test_construction_matches_reference_weights():
    from dwarf_v2_b200.model import EXPECTED_PARAMETERS, EXPECTED_TRAINABLE_PARAMETERS, DwarfConfig, DwarfForCausalLM

    g = load("model_prefill_b1_t2048")
    model = DwarfForCausalLM(DwarfConfig())
    assert sum(p.numel() for p in model.parameters()) == EXPECTED_PARAMETERS == int(g["param_count"])
    assert sum(p.numel() for p in model.parameters() if p.requires_grad) == EXPECTED_TRAINABLE_PARAMETERS
    digest = hashlib.sha256()
    for name, tensor in model.state_dict().items():
        digest.update(name.encode())
        digest.update(tensor.detach().float().numpy().tobytes())
    assert digest.digest() == bytes(g["param_sha256"].numpy().tolist())


def test_topology():
    from dwarf_v2_b200.model import DwarfForCausalLM, GlobalMixerBlock

    model = DwarfForCausalLM()
    kinds = ["HISA" if isinstance(b, GlobalMixerBlock) else "DSQG" for b in model.blocks]
    assert kinds == ["DSQG"] * 3 + ["HISA"] + ["DSQG"] * 6
    shifts = [b.attn.plane_shift for b in model.blocks if not isinstance(b, GlobalMixerBlock)]
    assert shifts == [0, 2, 4, 6, 8, 10, 12, 14, 0]
    assert [len(g) for g in model.offset_groups] == [29, 29, 29]
    assert model.lm_head.weight is model.embedding.weight


def test_forward_requires_cuda():
    from dwarf_v2_b200.model import DwarfForCausalLM

    model = DwarfForCausalLM()
    with pytest.raises(RuntimeError):
        model(torch.zeros(1, 8, dtype=torch.long))      # training mode, CPU tensor: no fallback
    with pytest.raises(RuntimeError):
        model.forward_lse(torch.zeros(1, 8, dtype=torch.long))
    model.eval()
    with torch.no_grad(), pytest.raises(RuntimeError):
        model(torch.zeros(1, 8, dtype=torch.long))      # CPU tensor: no fallback


def _err(out, ref):
    err = np.abs(np.asarray(out, np.float64) - np.asarray(ref, np.float64))
    return err.max(), err.mean() / np.abs(ref).mean()


@pytest.mark.gpu
@pytest.mark.parametrize("kv_cache", ["bf16", "q6"])
def test_prefill_matches_reference(kv_cache):
    from dwarf_v2_b200.model import DwarfForCausalLM

    g = load("model_prefill_b1_t2048")
    model = DwarfForCausalLM(kv_cache=kv_cache).eval().to(torch.bfloat16).cuda()
    ids = g["input_ids"].cuda()
    with torch.no_grad():
        logits = model(ids)[0, g["positions"].cuda()].float().cpu().numpy()
        logits2 = model(ids)[0, g["positions"].cuda()].float().cpu().numpy()
    assert np.array_equal(logits, logits2)  # deterministic
    f32 = g["logits_f32"].numpy()
    if kv_cache == "bf16":
        ref = g["logits_bf16"].numpy()
        ref_max, ref_mean = _err(ref, f32)
        mx, mean = _err(logits, f32)
        assert mx <= 1.5 * ref_max and mean <= 1.5 * ref_mean, (mx, mean, ref_max, ref_mean)
        mx, mean = _err(logits, ref)
        assert mx <= 0.08 and mean <= 0.025, (mx, mean)
    else:
        mx, mean = _err(logits, g["logits_bf16_q6"].numpy())
        assert mx <= 0.15 and mean <= 0.05, (mx, mean)


def test_cpu_oracle_matches_reference_fp32_logits():
    """oracle/model.py (the timed CPU baseline) reproduces the reference's fp32 logits."""
    from oracle import model as omodel

    from dwarf_v2_b200.dsqg_attention_v22 import ALL_OFFSETS
    from dwarf_v2_b200.model import DwarfForCausalLM

    g = load("model_prefill_b1_t2048")
    logits = omodel.prefill(DwarfForCausalLM().state_dict(), g["input_ids"], all_offsets=ALL_OFFSETS)
    err = np.abs(logits[0, g["positions"]].numpy() - g["logits_f32"].numpy())
    assert err.max() < 2e-3, err.max()


@pytest.mark.gpu
@pytest.mark.parametrize("kv_cache", ["bf16", "q6"])
def test_each_block_matches_the_reference_block_at_the_north_star_bar(kv_cache):
    """Teacher-forced per-block parity (reference train/train_dwarf.py:320-322 DSQG,
    :356-364 HISA; fixture tests/golden/model_blocks_b1_t2048.npz): every engine block
    gets the input its reference block got (seeded randn scaled to the RMS of that
    block's real input in the reference bf16 prefill, T=2048) and its output must be
    within 2e-2 max-abs and 1e-2 mean-relative of the reference bf16 block's output;
    on the q6 cache, of the reference block run on q6-round-tripped K/V. The computed
    part (output - input) must also stay within 2x the reference bf16 block's own
    error against its fp32 run (+ 2e-3), i.e. no worse than the reference's bf16 path."""
    from dwarf_v2_b200.model import DwarfForCausalLM

    g = load("model_blocks_b1_t2048")
    model = DwarfForCausalLM(kv_cache=kv_cache).eval().to(torch.bfloat16).cuda()
    rows = g["rows"]
    report = []
    with torch.no_grad():
        for i in range(len(model.blocks)):
            gen = torch.Generator().manual_seed(100 + i)
            xin = (torch.randn(1, 2048, 512, generator=gen) * float(g["input_rms"][i])).to(torch.bfloat16)
            out = model.prefill_block(i, xin.cuda())[0, rows.cuda()].float().cpu().numpy()
            key = f"block{i}_bf16_q6" if kv_cache == "q6" and f"block{i}_bf16_q6" in g else f"block{i}_bf16"
            ref = g[key].float().numpy()
            mx, mean = _err(out, ref)
            x0 = xin[0, rows].float().numpy()
            d_out, d_ref16, d_ref32 = out - x0, g[f"block{i}_bf16"].float().numpy() - x0, g[f"block{i}_f32"].numpy() - x0
            report.append((i, round(mx, 5), round(mean, 5)))
            assert mx <= 2e-2 and mean <= 1e-2, (kv_cache, i, mx, mean)
            if kv_cache == "bf16":
                e_out, e_ref = np.abs(d_out - d_ref32), np.abs(d_ref16 - d_ref32)
                assert e_out.max() <= 2 * e_ref.max() + 2e-3, (i, e_out.max(), e_ref.max())
                assert e_out.mean() <= 2 * e_ref.mean() + 2e-4, (i, e_out.mean(), e_ref.mean())
    print(kv_cache, report)


@pytest.mark.gpu
def test_prefill_graph_replays_the_eager_forward_bit_for_bit():
    """capture_prefill: one CUDA graph of the whole prefill (q6 KV) gives the eager
    forward's logits bit for bit, for two different inputs replayed in turn."""
    from dwarf_v2_b200.model import DwarfForCausalLM

    model = DwarfForCausalLM(kv_cache="q6").eval().to(torch.bfloat16).cuda()
    g = torch.Generator().manual_seed(3)
    ids = [torch.randint(57, 32768, (2, 320), generator=g).cuda() for _ in range(2)]
    with torch.no_grad():
        eager = [model(x).clone() for x in ids]
        graph = model.capture_prefill(2, 320)
        for x, ref in zip(ids * 2, eager * 2):
            assert torch.equal(graph(x), ref)
    with pytest.raises(ValueError):
        graph(ids[0][:, :100])
