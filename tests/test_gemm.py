"""tcgen05 GEMM with fused epilogues (dwarf_gemm_bf16) against torch fp32.

The reference computes every projection with nn.Linear in bf16
(train/train_dwarf.py:230-240, 299-364); the engine runs them on its own
tensor-core kernel. Checks: fp32-accumulated product within bf16 output
rounding (2 ulp), bias, ragged M and K, the SwiGLU epilogue against the
unfused linear + dwarf_swiglu path, and the up/gate interleaving (CPU).
"""

import pytest
import torch


def _ulps(out, ref):
    out, ref = out.float(), ref.float()
    ulp = torch.clamp(ref.abs(), min=1e-3) * 2.0 ** -7
    return ((out - ref).abs() / ulp).max().item()


def test_interleave_up_gate_layout():
    from dwarf_v2_b200.gemm import interleave_up_gate, swiglu_tile

    F, K = 1600, 8
    w = torch.arange(2 * F * K, dtype=torch.float32).reshape(2 * F, K)
    h = swiglu_tile(F)
    assert h == 80
    wi = interleave_up_gate(w)
    for t in (0, 7, F // h - 1):
        assert torch.equal(wi[2 * h * t:2 * h * t + h], w[h * t:h * (t + 1)])
        assert torch.equal(wi[2 * h * t + h:2 * h * (t + 1)], w[F + h * t:F + h * (t + 1)])


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K,bias", [
    (1000, 512, 512, None),
    (4096 + 77, 2048, 512, "f32"),
    (300, 256, 1600, "bf16"),
    (129, 128, 200, None),        # ragged K (zero-filled last k-block), N tile 128
    (20000, 512, 2048, None),     # many tiles per CTA (persistent loop, both accumulators)
])
def test_linear_matches_fp32(M, N, K, bias):
    from dwarf_v2_b200.gemm import linear

    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    b = None
    if bias == "f32":
        b = torch.randn(N, device="cuda", generator=g)
    elif bias == "bf16":
        b = torch.randn(N, device="cuda", generator=g).to(torch.bfloat16)
    out = linear(x, w, b)
    torch.cuda.synchronize()
    ref = x.float() @ w.float().T + (b.float() if b is not None else 0)
    assert _ulps(out, ref) <= 2.0
    assert torch.isfinite(out.float()).all()


@pytest.mark.gpu
@pytest.mark.parametrize("M,F,K", [(5000, 1600, 512), (333, 1024, 256), (128, 256, 64)])
def test_linear_swiglu_matches_unfused(M, F, K):
    from dwarf_v2_b200 import glue
    from dwarf_v2_b200.gemm import interleave_up_gate, linear_swiglu, swiglu_tile

    g = torch.Generator(device="cuda").manual_seed(F + K)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(2 * F, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    h = swiglu_tile(F)
    out = linear_swiglu(x, interleave_up_gate(w, h), h)
    torch.cuda.synchronize()
    ug = (x.float() @ w.float().T).to(torch.bfloat16)  # exact-product reference, bf16 like nn.Linear
    ref = glue.swiglu(ug)
    # bf16 inputs of silu/up may differ by one rounding from the fp32-exact product.
    assert _ulps(out, ref) <= 4.0
    err = (out.float() - ref.float()).abs()
    assert err.mean().item() <= 1e-3 * ref.float().abs().mean().item() + 1e-6


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K,wdtype,inplace", [
    (4096, 512, 512, torch.float32, False),
    (3000 + 5, 512, 1600, torch.bfloat16, True),
    (700, 256, 512, torch.float32, False),
])
def test_linear_add_rmsnorm_matches_unfused(M, N, K, wdtype, inplace):
    from dwarf_v2_b200 import glue
    from dwarf_v2_b200.gemm import linear, linear_add_rmsnorm

    g = torch.Generator(device="cuda").manual_seed(M + K)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    resid = (torch.randn(M, N, device="cuda", generator=g) * 2).to(torch.bfloat16)
    nw = (torch.rand(N, device="cuda", generator=g) + 0.5).to(wdtype)
    ref_x, ref_n = glue.add_rmsnorm(resid.clone(), nw, addend=linear(x, w))
    r_in = resid.clone()
    v, n = linear_add_rmsnorm(x, w, r_in, nw, x_out=r_in if inplace else None)
    torch.cuda.synchronize()
    assert torch.equal(v, ref_x)                   # same GEMM sums, same bf16 add
    if inplace:
        assert v.data_ptr() == r_in.data_ptr()
    assert _ulps(n, ref_n.float()) <= 1.0          # sum-of-squares order only
    assert (n != ref_n).float().mean().item() < 1e-3


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,heads", [(2, 2048, 8), (3, 200, 4)])
def test_qkvg_prep_matches_unfused(B, T, heads):
    import torch.nn.functional as F

    from dwarf_v2_b200.dsqg_attention_v22 import dsqg_prep
    from dwarf_v2_b200.gemm import linear, qkvg_prep

    D = 64 * heads
    g = torch.Generator(device="cuda").manual_seed(T + heads)
    x = torch.randn(B, T, D, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(4 * D, D, device="cuda", generator=g) / D ** 0.5).to(torch.bfloat16)
    bias = (torch.randn(4 * D, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    qp = F.normalize(torch.randn(4, 64, device="cuda", generator=g), dim=-1)
    kp = F.normalize(torch.randn(4, 64, device="cuda", generator=g), dim=-1)
    qkvg, y, z, (kc, ks, vc, vs) = qkvg_prep(x, w, bias, heads, qp, kp)
    torch.cuda.synchronize()
    ref = linear(x, w, bias)
    split = ref.view(B, T, 4, heads, 64)
    q, k, v = (split[:, :, i].permute(0, 2, 1, 3) for i in range(3))
    ry, rz, (rkc, rks, rvc, rvs) = dsqg_prep(q, k, v, qp, kp, pack_q6=True)
    assert torch.equal(qkvg[..., :D], ref[..., :D])
    assert torch.equal(qkvg[..., 3 * D:], ref[..., 3 * D:])
    assert torch.equal(kc, rkc) and torch.equal(vc, rvc)
    assert torch.equal(ks, rks) and torch.equal(vs, rvs)
    assert (y - ry).abs().max().item() < 1e-5
    assert (z - rz).abs().max().item() < 1e-5


@pytest.mark.gpu
def test_qkvg_prep_q6_codes_with_subnormal_scales():
    """Rows whose K/V amax is far below the fp16 normal range (zero inputs, bias ~1e-7):
    their fp16 scales are subnormal, the rounded scale can sit well below amax, and the
    codes depend on the clamp to +-31; they must still equal the unfused pack's."""
    import torch.nn.functional as F

    from dwarf_v2_b200.dsqg_attention_v22 import dsqg_prep
    from dwarf_v2_b200.gemm import linear, qkvg_prep

    B, T, heads = 2, 300, 4
    D = 64 * heads
    g = torch.Generator(device="cuda").manual_seed(17)
    x = torch.randn(B, T, D, device="cuda", generator=g).to(torch.bfloat16)
    x[:, ::3] = 0.0
    w = (torch.randn(4 * D, D, device="cuda", generator=g) / D ** 0.5).to(torch.bfloat16)
    bias = torch.randn(4 * D, device="cuda", generator=g) * 0.1
    bias[D:3 * D] = torch.randn(2 * D, device="cuda", generator=g) * 1e-7
    bias = bias.to(torch.bfloat16)
    qp = F.normalize(torch.randn(4, 64, device="cuda", generator=g), dim=-1)
    kp = F.normalize(torch.randn(4, 64, device="cuda", generator=g), dim=-1)
    _, _, _, (kc, ks, vc, vs) = qkvg_prep(x, w, bias, heads, qp, kp)
    ref = linear(x, w, bias).view(B, T, 4, heads, 64)
    q, k, v = (ref[:, :, i].permute(0, 2, 1, 3) for i in range(3))
    _, _, (rkc, rks, rvc, rvs) = dsqg_prep(q, k, v, qp, kp, pack_q6=True)
    assert bool((rks[:, :, ::3].float() < 6.1e-5).all())  # the zero rows have subnormal scales
    assert torch.equal(kc, rkc) and torch.equal(vc, rvc)
    assert torch.equal(ks, rks) and torch.equal(vs, rvs)
