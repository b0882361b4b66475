"""Weights from the reference's checkpoints.

Mirrors the model half of ``restore_checkpoint`` (train/train_dwarf.py:976-1018)
for a forward engine. Two sources:

* a ``dwarf-55m-resume-v1`` payload written by ``checkpoint_payload``
  (:954-973) is held to the reference's own checks, in its order: the payload
  kind, then the saved key set against ``model.state_dict()`` (no migration:
  the reference compares keys before loading), then every tensor's shape AND
  dtype (:997-1002); any mismatch raises ``ValueError`` with the reference's
  message and nothing is loaded. So a bf16 engine model takes a resume payload
  only after ``model.float()`` (the reference trains and saves fp32), or with
  ``cast=True``;
* a bare model state dict (not a reference format: e.g. the modules' older
  key layouts) first goes through the modules' legacy-key migrations (DSQG
  ``qkv_proj``/``gate_proj``/``pos_bias``; HISA ``W_q``/``W_k``/``W_v``), then
  the key, shape and dtype checks.

``cast=True`` relaxes only the dtype check: values are cast to the model's
dtype on load. Optimizer, RNG, recipe and dataset identity are training-side
and are not restored.
"""

from __future__ import annotations

from pathlib import Path
from typing import Any

import torch

KIND = "dwarf-55m-resume-v1"


def _payload(source: str | Path | dict[str, Any]) -> tuple[dict[str, torch.Tensor], bool]:
    """(model state dict, is_resume_payload) of a payload (path or loaded dict) or a bare state dict."""
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
        return state, True
    if source and all(torch.is_tensor(v) for v in source.values()):
        return source, False
    raise ValueError("not a 55M DWARF resumable checkpoint")


def model_state_from(source: str | Path | dict[str, Any]) -> dict[str, torch.Tensor]:
    """The model state dict of a payload (path or loaded dict) or a bare state dict."""
    return _payload(source)[0]


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


def load_weights(model: torch.nn.Module, source: str | Path | dict[str, Any], *, cast: bool = False) -> None:
    """Validates, then strictly loads, reference weights into ``model``.

    Raises ``ValueError`` with the reference's messages when the payload kind, the
    key set, a tensor shape or (unless ``cast``) a tensor dtype does not match;
    nothing is loaded in that case.
    """
    state, resume = _payload(source)
    staged = dict(state) if resume else migrate_legacy_keys(model, state)
    expected = model.state_dict()
    if staged.keys() != expected.keys():
        raise ValueError("checkpoint model keys do not match")
    for name, ref in expected.items():
        got = staged[name]
        if not torch.is_tensor(got) or got.shape != ref.shape or (got.dtype != ref.dtype and not cast):
            raise ValueError(f"checkpoint model tensor does not match: {name}")
    with torch.no_grad():
        model.load_state_dict(staged, strict=True)
