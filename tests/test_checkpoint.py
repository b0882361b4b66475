"""Weights from the reference's checkpoints (CPU).

Legacy-key migration pinned to the reference's own _load_from_state_dict
(dsqg_attention_v22.py:3069-3142, hierarchical_sparse_attn_v18_hisa.py:2469-2544)
through tests/golden/checkpoint_*_legacy.npz, and the payload validation of
restore_checkpoint (train/train_dwarf.py:976-1018).
"""

import pytest
import torch

from tests._golden import load


def _split(g, prefix):
    return {k[len(prefix):]: v for k, v in g.items() if k.startswith(prefix)}


def test_dsqg_legacy_keys_match_reference_migration():
    from dwarf_v2_b200.dsqg_attention_v22 import DSQGAttentionV19

    g = load("checkpoint_dsqg_legacy")
    legacy, loaded = _split(g, "legacy."), _split(g, "loaded.")
    module = DSQGAttentionV19(128, 2, [1, 2, 3, 5, 8, 13, 21, 48, 64, 100], 7, 3, seq_len=160, dropout=0.0,
                              plane_shift=6)
    module.load_state_dict({k: v.clone() for k, v in legacy.items()}, strict=True)
    state = module.state_dict()
    assert state.keys() == loaded.keys()
    for key, ref in loaded.items():
        assert torch.equal(state[key].reshape(-1), ref.reshape(-1)), key  # fixtures store 0-d as 1-d


def test_hisa_legacy_keys_match_reference_migration():
    from dwarf_v2_b200.hierarchical_sparse_attn_v18_hisa import HierarchicalSparseAttentionV16HISACausal

    g = load("checkpoint_hisa_legacy")
    legacy, loaded = _split(g, "legacy."), _split(g, "loaded.")
    module = HierarchicalSparseAttentionV16HISACausal(
        D=128, H=2, hd=64, chunk_size=64, top_k_chunks=4, hisa_top_m_tokens=64, local_window=64,
        selector_tile_size=16, representative_mode="mean_max_blend", representative_blend_alpha=0.5,
        route_prior_scale=0.1, global_adapter_rank=16, npci_theta_max=0.25, local_backend="flex")
    before = {k: v.clone() for k, v in module.state_dict().items()}
    block = torch.nn.Module()  # the block owning the legacy gate_proj
    block.attn = module
    result = block.load_state_dict({k: v.clone() for k, v in legacy.items()}, strict=False)
    assert not result.missing_keys
    after = module.state_dict()
    for key in ("qkvg_proj.weight", "qkvg_proj.bias", "W_o.weight", "route_prior_raw", "npci_theta_k",
                "npci_theta_v", "global_k_up.weight", "global_v_up.weight"):
        assert torch.equal(after[key], loaded[key]), key
    # randomly initialised parameters newer than the checkpoint keep this module's values
    for key in ("global_k_down.weight", "global_v_down.weight"):
        assert torch.equal(after[key], before[key]), key


def test_model_payload_round_trip_and_validation():
    from dwarf_v2_b200.checkpoint import KIND, load_weights
    from dwarf_v2_b200.model import DwarfConfig, DwarfForCausalLM

    src = DwarfForCausalLM(DwarfConfig(init_seed=7))
    dst = DwarfForCausalLM()
    payload = {"kind": KIND, "step": 10, "model": src.state_dict()}
    load_weights(dst, payload)
    for (k, a), (_, b) in zip(src.state_dict().items(), dst.state_dict().items()):
        assert torch.equal(a, b), k
    snapshot = {k: v.clone() for k, v in dst.state_dict().items()}
    with pytest.raises(ValueError, match="not a 55M DWARF resumable checkpoint"):
        load_weights(dst, {"kind": "something-else", "model": src.state_dict()})
    broken = dict(src.state_dict())
    broken.pop("norm.weight")
    with pytest.raises(ValueError, match="keys do not match"):
        load_weights(dst, {"kind": KIND, "model": broken})
    wrong = dict(src.state_dict())
    wrong["norm.weight"] = torch.zeros(3)
    with pytest.raises(ValueError, match="tensor does not match: norm.weight"):
        load_weights(dst, {"kind": KIND, "model": wrong})
    for k, v in dst.state_dict().items():  # nothing was loaded by the failed calls
        assert torch.equal(v, snapshot[k]), k


def test_resume_payload_is_held_to_the_reference_checks():
    """A dwarf-55m-resume-v1 payload: a tensor whose dtype differs from the model's is
    refused (restore_checkpoint, train/train_dwarf.py:999-1002) unless cast=True; a
    stray key and a legacy-layout key are refused before any migration (the reference
    compares the key sets first, :996-997); a bare state dict still migrates legacy keys."""
    from dwarf_v2_b200.checkpoint import KIND, load_weights
    from dwarf_v2_b200.model import DwarfConfig, DwarfForCausalLM

    src = DwarfForCausalLM(DwarfConfig(init_seed=3))
    dst = DwarfForCausalLM()
    snapshot = {k: v.clone() for k, v in dst.state_dict().items()}
    half = {k: v.to(torch.bfloat16) if v.is_floating_point() else v for k, v in src.state_dict().items()}
    with pytest.raises(ValueError, match="tensor does not match"):
        load_weights(dst, {"kind": KIND, "model": half})
    stray = dict(src.state_dict())
    stray["blocks.0.attn.not_a_parameter"] = torch.zeros(1)
    with pytest.raises(ValueError, match="keys do not match"):
        load_weights(dst, {"kind": KIND, "model": stray})
    legacy = dict(src.state_dict())
    legacy["blocks.0.attn.qkv_proj.weight"] = legacy.pop("blocks.0.attn.qkvg_proj.weight")
    with pytest.raises(ValueError, match="keys do not match"):
        load_weights(dst, {"kind": KIND, "model": legacy})
    for k, v in dst.state_dict().items():  # nothing was loaded by the refused payloads
        assert torch.equal(v, snapshot[k]), k
    load_weights(dst, {"kind": KIND, "model": half}, cast=True)
    for k, v in dst.state_dict().items():
        assert torch.equal(v, half[k].to(v.dtype)), k
