"""Fused lm_head + cross entropy (forward), without materialising logits.

Mirrors the loss the reference trainer builds and calls
(train/train_dwarf.py:1084 ``LigerFusedLinearCrossEntropyLoss(accum_dtype=
torch.float32)``; :1134-1138 ``loss_fn(model.lm_head.weight, hidden.flatten(0, 1),
labels.flatten())``): the mean over non-ignored labels of
``logsumexp(l) - l[label]`` where ``l = bf16(hidden @ weight.T)`` is upcast to
fp32. On B200 the lm_head GEMM reduces the logits in its epilogue
(``gemm.linear_lse``); nothing of size [rows, vocab] is written.

Forward (inference / evaluation) only: this loss has no backward here. Training
runs the reference's own loss formula over the model's differentiable path.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from . import gemm


def fused_linear_cross_entropy(weight: torch.Tensor, hidden: torch.Tensor, target: torch.Tensor, *,
                               ignore_index: int = -100, reduction: str = "mean") -> torch.Tensor:
    if reduction not in ("mean", "sum", "none"):
        raise ValueError(f"reduction must be 'mean', 'sum' or 'none', got {reduction!r}")
    if torch.is_grad_enabled() and (weight.requires_grad or hidden.requires_grad):
        raise NotImplementedError("dwarf_v2_b200 is a forward (inference) engine; run under torch.no_grad()")
    if hidden.ndim != 2 or target.ndim != 1 or target.shape[0] != hidden.shape[0]:
        raise ValueError("expected hidden [rows, D] and target [rows]")
    act = torch.bfloat16
    _, _, loss = gemm.linear_lse(hidden.to(act), weight.detach().to(act), target, ignore_index=ignore_index)
    if reduction == "none":
        return loss
    total = loss.sum()
    if reduction == "sum":
        return total
    return total / (target != ignore_index).sum().clamp_min(1).to(total.dtype)


class FusedLinearCrossEntropyLoss(nn.Module):
    """``LigerFusedLinearCrossEntropyLoss``'s forward: ``loss(lin_weight, _input, target, bias=None)``."""

    def __init__(self, accum_dtype: torch.dtype | None = None, ignore_index: int = -100, reduction: str = "mean",
                 **unsupported) -> None:
        super().__init__()
        for key, value in unsupported.items():
            neutral = {"lse_square_scale": 0.0, "label_smoothing": 0.0, "softcap": None, "return_z_loss": False}
            if key not in neutral or value != neutral[key]:
                raise NotImplementedError(f"option {key}={value!r} is not implemented by the B200 engine")
        self.accum_dtype = accum_dtype  # gradient accumulation dtype in the reference; no backward here
        self.ignore_index = int(ignore_index)
        self.reduction = reduction

    def forward(self, lin_weight: torch.Tensor, _input: torch.Tensor, target: torch.Tensor,
                bias: torch.Tensor | None = None) -> torch.Tensor:
        if bias is not None:
            raise NotImplementedError("the B200 lm_head has no bias")
        return fused_linear_cross_entropy(lin_weight, _input, target, ignore_index=self.ignore_index,
                                          reduction=self.reduction)


LigerFusedLinearCrossEntropyLoss = FusedLinearCrossEntropyLoss
