"""Fused lm_head + logsumexp / argmax / cross entropy (the forward of the
reference trainer's LigerFusedLinearCrossEntropyLoss, train/train_dwarf.py:1084,
1134-1138) against torch on the logits the plain lm_head GEMM writes.

Tolerances: argmax bit-exact (same fp32 accumulators, same bf16 rounding, first
index on ties, as torch.argmax); lse and per-token loss within 1e-4 abs (the
epilogue sums exp2 on the SFU, fp32).
"""

import pytest
import torch


def test_loss_module_rejects_unsupported_options():
    from dwarf_v2_b200.fused_linear_cross_entropy import LigerFusedLinearCrossEntropyLoss

    LigerFusedLinearCrossEntropyLoss(accum_dtype=torch.float32, label_smoothing=0.0)
    with pytest.raises(NotImplementedError):
        LigerFusedLinearCrossEntropyLoss(label_smoothing=0.1)
    with pytest.raises(ValueError):
        from dwarf_v2_b200.fused_linear_cross_entropy import fused_linear_cross_entropy
        fused_linear_cross_entropy(torch.zeros(4, 2), torch.zeros(3, 2), torch.zeros(3), reduction="avg")


@pytest.mark.gpu
@pytest.mark.parametrize("M,N", [(1000, 32768), (256, 512), (37, 1024), (3000, 4096)])
def test_linear_lse_matches_logits(M, N):
    from dwarf_v2_b200 import gemm

    g = torch.Generator().manual_seed(M + N)
    x = torch.randn(M, 512, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(N, 512, generator=g) * 0.05).to(torch.bfloat16).cuda()
    w[7] = w[3]  # duplicate rows: exact ties in every row's logits
    t = torch.randint(0, N, (M,), generator=g).cuda()
    t[::5] = -100
    lse, am, loss = gemm.linear_lse(x, w, t)
    logits = gemm.linear(x, w).float()
    torch.cuda.synchronize()
    ref_lse = torch.logsumexp(logits, -1)
    torch.testing.assert_close(lse, ref_lse, atol=1e-4, rtol=0)
    assert torch.equal(am, logits.argmax(-1))
    ref_loss = torch.nn.functional.cross_entropy(logits, t, ignore_index=-100, reduction="none")
    torch.testing.assert_close(loss, ref_loss, atol=1e-4, rtol=0)
    lse2, am2, none = gemm.linear_lse(x, w)
    assert none is None and torch.equal(lse2, lse) and torch.equal(am2, am)


@pytest.mark.gpu
@torch.no_grad()
def test_model_loss_matches_full_logits():
    from dwarf_v2_b200.fused_linear_cross_entropy import LigerFusedLinearCrossEntropyLoss
    from dwarf_v2_b200.model import DwarfForCausalLM

    model = DwarfForCausalLM(kv_cache="q6").eval().to(torch.bfloat16).cuda()
    g = torch.Generator().manual_seed(2)
    batch = torch.randint(57, 32768, (2, 513), generator=g).cuda()
    input_ids, labels = batch[:, :-1], batch[:, 1:]
    hidden = model(input_ids, return_hidden=True)
    loss = LigerFusedLinearCrossEntropyLoss(accum_dtype=torch.float32)(
        model.lm_head.weight, hidden.flatten(0, 1), labels.flatten())
    logits = model(input_ids).float()
    ref = torch.nn.functional.cross_entropy(logits.flatten(0, 1), labels.flatten())
    torch.testing.assert_close(loss, ref, atol=1e-4, rtol=0)


@pytest.mark.gpu
@torch.no_grad()
def test_model_forward_lse_matches_logits():
    from dwarf_v2_b200.model import DwarfForCausalLM

    model = DwarfForCausalLM(kv_cache="q6").eval().to(torch.bfloat16).cuda()
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(57, 32768, (2, 300), generator=g).cuda()
    labels = torch.randint(57, 32768, (2, 300), generator=g).cuda()
    lse, am, loss = model.forward_lse(ids, labels)
    logits = model(ids).float()
    torch.testing.assert_close(lse, torch.logsumexp(logits, -1), atol=1e-4, rtol=0)
    assert torch.equal(am, logits.argmax(-1))
    ref = torch.nn.functional.cross_entropy(logits.flatten(0, 1), labels.flatten(), reduction="none")
    torch.testing.assert_close(loss.flatten(), ref, atol=1e-4, rtol=0)
