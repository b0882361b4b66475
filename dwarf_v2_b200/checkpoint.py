"""Weights from the reference's checkpoints.

Mirrors the model half of ``restore_checkpoint`` (train/train_dwarf.py:976-1018)
for a forward engine: the ``dwarf-55m-resume-v1`` payload written by
``checkpoint_payload`` (:954-973) -- or a bare model state dict -- is validated
(kind, key set, tensor shapes) and loaded strictly. Optimizer, RNG, recipe and
dataset identity are training-side and are not restored. Older key layouts are
migrated by the modules' own ``_load_from_state_dict`` hooks (DSQG
``qkv_proj``/``gate_proj``/``pos_bias``; HISA ``W_q``/``W_k``/``W_v``).
"""

from __future__ import annotations

from pathlib import Path
from typing import Any

import torch

KIND = "dwarf-55m-resume-v1"


def model_state_from(source: str | Path | dict[str, Any]) -> dict[str, torch.Tensor]:
    """The model state dict of a payload (path or loaded dict) or a bare state dict."""
    if isinstance(source, (str, Path)):
        source = torch.load(Path(source), map_location="cpu", weights_only=True)
    if not isinstance(source, dict):
        raise ValueError("not a 55M DWARF resumable checkpoint")
    if "kind" in source:
        if source.get("kind") != KIND:
            raise ValueError("not a 55M DWARF resumable checkpoint")
        state = source.get("model")
        if not isinstance(state, dict):
            raise ValueError("checkpoint model keys do not match")
        return state
    if source and all(torch.is_tensor(v) for v in source.values()):
        return source
    raise ValueError("not a 55M DWARF resumable checkpoint")


def migrate_legacy_keys(model: torch.nn.Module, state: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    """A copy of ``state`` with every module's legacy keys rewritten (nothing is loaded)."""
    staged = dict(state)

    def walk(module: torch.nn.Module, prefix: str) -> None:
        migrate = getattr(module, "_migrate_legacy_keys", None)
        if migrate is not None:
            migrate(staged, prefix)
        for name, child in module._modules.items():
            if child is not None:
                walk(child, prefix + name + ".")

    walk(model, "")
    return staged


def load_weights(model: torch.nn.Module, source: str | Path | dict[str, Any]) -> None:
    """Validates, then strictly loads, reference weights into ``model`` (values cast to its dtype/device).

    Raises ``ValueError`` with the reference's messages when the payload kind, the
    key set or a tensor shape does not match; nothing is loaded in that case.
    """
    staged = migrate_legacy_keys(model, model_state_from(source))
    expected = model.state_dict()
    if staged.keys() != expected.keys():
        raise ValueError("checkpoint model keys do not match")
    for name, ref in expected.items():
        got = staged[name]
        if not torch.is_tensor(got) or got.shape != ref.shape:
            raise ValueError(f"checkpoint model tensor does not match: {name}")
    with torch.no_grad():
        model.load_state_dict(staged, strict=True)
