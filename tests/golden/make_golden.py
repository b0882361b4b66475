"""Generates the golden fixtures in tests/golden/ by running the REFERENCE code.

Run where a checkout of the reference exists, with its path in the required
environment variable DWARF_REFERENCE_DIR; the fixtures it writes are committed
and the tests read only those files, so nothing at test time needs the reference.

    DWARF_REFERENCE_DIR=<checkout> python tests/golden/make_golden.py [ema|dsqg|hisa|model|model_blocks|checkpoint|all]

Each fixture is an ``.npz`` holding the seeded inputs and the reference output
of one call, named for the reference function it exercises. bf16 tensors are
stored as their uint16 bit patterns (key suffix ``__bf16``).
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
REFERENCE = Path(os.environ["DWARF_REFERENCE_DIR"]) if os.environ.get("DWARF_REFERENCE_DIR") else None


def _import_reference():
    if REFERENCE is None or not (REFERENCE / "kernels").is_dir():
        raise SystemExit("set DWARF_REFERENCE_DIR to a checkout of the reference (kernels/, train/)")
    for sub in ("kernels", "train"):
        path = str(REFERENCE / sub)
        if path not in sys.path:
            sys.path.insert(0, path)


def to_np(tensor: torch.Tensor) -> tuple[str, np.ndarray]:
    tensor = tensor.detach().cpu()
    if tensor.dtype == torch.bfloat16:
        return "__bf16", tensor.view(torch.int16).numpy().view(np.uint16)
    return "", tensor.numpy()


def save(name: str, **arrays) -> None:
    out = {}
    for key, value in arrays.items():
        if isinstance(value, torch.Tensor):
            suffix, arr = to_np(value)
            out[key + suffix] = arr
        else:
            out[key] = np.asarray(value)
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print("wrote", name, {k: v.shape for k, v in out.items()})


def make_ema() -> None:
    _import_reference()
    import causal_ema_scan as ref

    # The reference's own __main__ case (causal_ema_scan.py:570-581), forward only.
    torch.manual_seed(1)
    x = torch.randn(2, 9, 7, dtype=torch.float64)
    raw = torch.tensor(ref.inverse_bounded_ema_factor(0.05), dtype=torch.float64)
    alpha = ref.bounded_ema_factor(raw)
    y = ref.causal_ema_scan(x, alpha)
    save("ema_reference_main_f64", x=x, alpha=alpha.reshape(1), y=y)

    # fp32, alpha above the ceiling (clamped to 0.5), ragged sizes.
    g = torch.Generator().manual_seed(11)
    x = torch.randn(3, 200, 96, generator=g, dtype=torch.float32)
    alpha = torch.tensor([0.7], dtype=torch.float32)
    y = ref.causal_ema_scan(x, alpha)
    save("ema_scalar_clamped_f32", x=x, alpha=alpha, y=y)

    # bf16 input as the model feeds it (train_dwarf.py:261), alpha = 1/16.
    g = torch.Generator().manual_seed(12)
    x = torch.randn(2, 130, 512, generator=g).to(torch.bfloat16)
    alpha = torch.tensor([1.0 / 16.0], dtype=torch.float32)
    y = ref.causal_ema_scan(x, alpha)
    save("ema_scalar_bf16", x=x, alpha=alpha, y=y)

    # Per-channel decay (y_t = a*y_{t-1} + (1-a)*x_t, a = sigmoid(N(0,1))): the
    # reference _reference broadcasts a [D] alpha, so alpha = 1-a with bounds
    # that never bind reproduces it.
    g = torch.Generator().manual_seed(13)
    x = torch.randn(2, 300, 64, generator=g, dtype=torch.float32)
    decay = torch.sigmoid(torch.randn(64, generator=g))
    y = ref._reference(x, 1.0 - decay, 1e-12, 1.0 - 1e-12)
    save("ema_per_channel_f32", x=x, decay=decay, y=y)


def make_ema_backward() -> None:
    """Backward golden vectors: autograd through the reference's own oracle
    ``_reference`` (kernels/causal_ema_scan.py:511-538), the function the
    reference's gradcheck (:570-581) validates its kernels against."""
    _import_reference()
    import causal_ema_scan as ref

    def grads(x, alpha, dy, floor, ceiling):
        x = x.clone().requires_grad_(True)
        alpha = alpha.clone().requires_grad_(True)
        y = ref._reference(x, alpha, floor, ceiling)
        dx, da = torch.autograd.grad(y, (x, alpha), dy)
        return y.detach(), dx, da

    # The reference __main__ shape, fp64, alpha = 0.05 inside the bounds.
    torch.manual_seed(1)
    x = torch.randn(2, 9, 7, dtype=torch.float64)
    alpha = ref.bounded_ema_factor(torch.tensor(ref.inverse_bounded_ema_factor(0.05), dtype=torch.float64))
    alpha = alpha.reshape(1)
    dy = torch.randn(2, 9, 7, dtype=torch.float64)
    y, dx, da = grads(x, alpha, dy, 1e-5, 0.5)
    save("ema_bwd_scalar_f64", x=x, alpha=alpha, dy=dy, y=y, dx=dx, da=da)

    # fp32, ragged sizes, alpha = 1/64 (the model's second packet scale).
    g = torch.Generator().manual_seed(21)
    x = torch.randn(3, 200, 96, generator=g, dtype=torch.float32)
    dy = torch.randn(3, 200, 96, generator=g, dtype=torch.float32)
    alpha = torch.tensor([1.0 / 64.0], dtype=torch.float32)
    y, dx, da = grads(x, alpha, dy, 1e-5, 0.5)
    save("ema_bwd_scalar_f32", x=x, alpha=alpha, dy=dy, y=y, dx=dx, da=da)

    # Per-channel alpha = 1 - sigmoid(N(0,1)) with bounds that never bind.
    g = torch.Generator().manual_seed(22)
    x = torch.randn(2, 300, 64, generator=g, dtype=torch.float32)
    dy = torch.randn(2, 300, 64, generator=g, dtype=torch.float32)
    alpha = 1.0 - torch.sigmoid(torch.randn(64, generator=g))
    y, dx, da = grads(x, alpha, dy, 1e-12, 1.0 - 1e-12)
    save("ema_bwd_per_channel_f32", x=x, alpha=alpha, dy=dy, y=y, dx=dx, da=da)


def _dsqg_case(module, q, k, v):
    """Reference tables + probe projections exactly as DSQGAttentionV19.forward builds them."""
    import torch.nn.functional as F

    gate = torch.sigmoid(module.phase_gate)[:, None, None]
    qp = F.normalize(module.query_probes.float(), dim=-1)
    kp = F.normalize(module.key_probes.float(), dim=-1)
    eps = 1e-6 * q.shape[-1]
    qf, kf = q.float(), k.float()
    y = torch.einsum("bhnd,rd->bhnr", qf, qp) * torch.rsqrt(qf.square().sum(-1, keepdim=True) + eps)
    z = torch.einsum("bhnd,rd->bhnr", kf, kp) * torch.rsqrt(kf.square().sum(-1, keepdim=True) + eps)
    return dict(
        pos_bias=module.pos_bias.detach().float(),
        scale_embed=module.centered_scale_embed.detach().float(),
        phase_base=(module.phase_base * gate).detach().float(),
        phase_gain=(module.phase_gain * gate).detach().float(),
        y_pre=y.detach(), z_pre=z.detach(),
        offsets=module.offsets_dev.clone(),
    )


def _randomize_dsqg(module, seed):
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        module.pos_bias_residual.copy_(torch.randn(module.pos_bias_residual.shape, generator=g) * 0.3)
        module.scale_embed.copy_(torch.randn(module.scale_embed.shape, generator=g) * 0.3)
        module.phase_base.copy_(torch.randn(module.phase_base.shape, generator=g) * 0.7)
        module.phase_gain.copy_(torch.randn(module.phase_gain.shape, generator=g) * 3.0)
        module.phase_gate.copy_(torch.randn(module.phase_gate.shape, generator=g))


def _triton_interpret_dsqg(case: dict, q, k, v, j_small, j_large, plane_shift, query_start):
    """Run the reference Triton kernel _fwd_v22_online on CPU under TRITON_INTERPRET=1."""
    import subprocess
    import tempfile

    with tempfile.TemporaryDirectory() as tmp:
        torch.save(dict(case=case, q=q, k=k, v=v, j_small=j_small, j_large=j_large,
                        plane_shift=plane_shift, query_start=query_start), f"{tmp}/in.pt")
        code = f"""
import sys, torch
sys.path.insert(0, {str(REFERENCE / 'kernels')!r})
import dsqg_attention_v22 as ref
d = torch.load({tmp!r} + '/in.pt')
c = d['case']; q, k, v = d['q'], d['k'], d['v']
B, H, N, HD = q.shape
out = torch.zeros_like(q); lse = torch.full((B, H, N), float('-inf'))
pb, se = c['pos_bias'].contiguous(), c['scale_embed'].contiguous()
ph, pg = c['phase_base'].contiguous(), c['phase_gain'].contiguous()
y, z = c['y_pre'].contiguous(), c['z_pre'].contiguous()
qs = d['query_start']
grid = (B * H, ref.triton.cdiv(max(0, N - qs), 64))
ref._fwd_v22_online[grid](q, k, v, pb, se, ph, pg, y, z, out, lse, c['offsets'],
    *q.stride(), *k.stride(), *v.stride(), *out.stride(), *lse.stride(), *pb.stride(), *se.stride(),
    *ph.stride()[:2], *pg.stride()[:2], *y.stride()[:3], *z.stride()[:3],
    H=H, N=N, HD=HD, BLOCK_N=64, BLOCK_HD=64, J_VAL=d['j_small'] + d['j_large'], J_SMALL_VAL=d['j_small'],
    J_LARGE_VAL=d['j_large'], R_PLANES_VAL=4, PLANE_SHIFT=d['plane_shift'], K_GROUP_SIZE=3,
    KV_HEAD_GROUP_SIZE=H // k.shape[1], QUERY_START=qs)
torch.save(dict(out=out, lse=lse), {tmp!r} + '/out.pt')
"""
        env = dict(os.environ, TRITON_INTERPRET="1")
        subprocess.run([sys.executable, "-c", code], check=True, env=env)
        return torch.load(f"{tmp}/out.pt")


def make_dsqg(with_triton: bool = True) -> None:
    _import_reference()
    import dsqg_attention_v22 as ref

    # B=1, H=8, hd=64, T=256, canonical 96-offset lattice.
    torch.manual_seed(1)
    module = ref.DSQGAttentionV19(512, 8, ref.ALL_OFFSETS, 17, 79, seq_len=2048, grouped_mode="baseline")
    _randomize_dsqg(module, 101)
    torch.manual_seed(0)
    q = torch.randn(1, 8, 256, 64).to(torch.bfloat16)
    k = torch.randn(1, 8, 256, 64).to(torch.bfloat16)
    v = torch.randn(1, 8, 256, 64).to(torch.bfloat16)
    case = _dsqg_case(module, q, k, v)
    eager = ref._eager_dsqg_attention(q.float(), k.float(), v.float(), case["pos_bias"], case["scale_embed"],
                                      case["phase_base"], case["phase_gain"], case["y_pre"], case["z_pre"],
                                      case["offsets"], 17, plane_shift=0)
    extra = {}
    if with_triton:
        tri = _triton_interpret_dsqg(case, q, k, v, 17, 79, 0, 1)
        extra = dict(triton_out=tri["out"], triton_lse=tri["lse"])
    save("dsqg_config1", q=q, k=k, v=v, eager_out=eager, j_small=17, j_large=79, plane_shift=0,
         query_start=1, **case, **extra)

    # GQA (H=4, H_kv=2), plane shift 10, ragged N, query_start past the minimum offset.
    torch.manual_seed(2)
    offsets = [1, 3, 7, 12, 28, 48, 50, 77, 130, 200]
    module = ref.DSQGAttentionV19(256, 4, offsets, 5, 5, seq_len=256, plane_shift=10)
    _randomize_dsqg(module, 202)
    q = torch.randn(2, 4, 157, 64).to(torch.bfloat16)
    k = torch.randn(2, 2, 157, 64).to(torch.bfloat16)
    v = torch.randn(2, 2, 157, 64).to(torch.bfloat16)
    case = _dsqg_case(module, q, k, v)
    case["z_pre"] = case["z_pre"]  # computed from the 2 KV heads
    eager = ref._eager_dsqg_attention(q.float(), k.float(), v.float(), case["pos_bias"], case["scale_embed"],
                                      case["phase_base"], case["phase_gain"], case["y_pre"], case["z_pre"],
                                      case["offsets"], 5, plane_shift=10)
    extra = {}
    if with_triton:
        tri = _triton_interpret_dsqg(case, q, k, v, 5, 5, 10, 1)
        extra = dict(triton_out=tri["out"], triton_lse=tri["lse"])
    save("dsqg_gqa_ragged", q=q, k=k, v=v, eager_out=eager, j_small=5, j_large=5, plane_shift=10,
         query_start=1, **case, **extra)

    # Whole module (eval, fp32 reference on bf16-valued inputs), head_dim 64.
    torch.manual_seed(3)
    module = ref.DSQGAttentionV19(128, 2, [1, 2, 3, 5, 8, 13, 21, 48, 64, 100], 7, 3, seq_len=160,
                                  dropout=0.0, plane_shift=6).eval()
    _randomize_dsqg(module, 303)
    with torch.no_grad():
        module.if_gain.copy_(torch.tensor([0.7, 1.3]))
    x = torch.randn(2, 150, 128).to(torch.bfloat16).float()
    with torch.no_grad():
        y = module(x)
    state = {f"state.{k}": val for k, val in module.state_dict().items()}
    save("dsqg_module_eval", x=x, y=y, **state)


def make_dsqg_backward() -> None:
    """Backward golden vectors: fp64 autograd through the reference's own eager
    oracle ``_eager_dsqg_attention`` (kernels/dsqg_attention_v22.py:2602-2688)
    on the inputs of the committed forward fixtures, with a seeded dO."""
    _import_reference()
    import dsqg_attention_v22 as ref

    sys.path.insert(0, str(HERE.parent.parent))
    from tests._golden import load

    names = ("q", "k", "v", "pos_bias", "scale_embed", "phase_base", "phase_gain", "y_pre", "z_pre")
    for src, dst, seed in (("dsqg_config1", "dsqg_bwd_config1", 31), ("dsqg_gqa_ragged", "dsqg_bwd_gqa_ragged", 32)):
        g = load(src)
        leaves = {n: g[n].double().clone().requires_grad_(True) for n in names}
        out = ref._eager_dsqg_attention(*(leaves[n] for n in names), g["offsets"], int(g["j_small"]),
                                        plane_shift=int(g["plane_shift"]))
        dout = torch.randn(out.shape, generator=torch.Generator().manual_seed(seed), dtype=torch.float64)
        dout = dout.to(torch.bfloat16)
        grads = torch.autograd.grad(out, [leaves[n] for n in names], dout.double())
        save(dst, dout=dout, out=out.detach().float(), **{f"d_{n}": gr.float() for n, gr in zip(names, grads)})


def make_dsqg_module_grad() -> None:
    """Training-mode gradients of the reference DSQGAttentionV19 (CPU, fp32 eager
    path, dropout 0): every parameter's gradient and dx for a seeded dy, with
    and without a kv_inject packet (NPCI path)."""
    _import_reference()
    import dsqg_attention_v22 as ref

    torch.manual_seed(4)
    module = ref.DSQGAttentionV19(128, 2, [1, 2, 3, 5, 8, 13, 21, 48, 64, 100], 7, 3, seq_len=160,
                                  dropout=0.0, plane_shift=6).train()
    _randomize_dsqg(module, 404)
    g = torch.Generator().manual_seed(405)
    x = torch.randn(2, 150, 128, generator=g).to(torch.bfloat16).float()
    kd = torch.randn(2, 2, 150, 64, generator=g) * 0.5
    vd = torch.randn(2, 2, 150, 64, generator=g) * 0.5
    dy = torch.randn(2, 150, 128, generator=g)
    state = {f"state.{k}": val for k, val in module.state_dict().items()}
    out = {}
    for tag, inject in (("plain", None), ("inject", (kd, vd))):
        module.zero_grad()
        xl = x.clone().requires_grad_(True)
        y = module(xl, inject)
        y.backward(dy)
        out[f"{tag}.y"] = y.detach()
        out[f"{tag}.dx"] = xl.grad
        for name, p in module.named_parameters():
            if p.grad is not None:
                out[f"{tag}.grad.{name}"] = p.grad.clone()
    save("dsqg_module_grad", x=x, kd=kd, vd=vd, dy=dy, **state, **out)


def make_hisa() -> None:
    _import_reference()
    import torch.nn.functional as F

    import hierarchical_sparse_attn_v18_hisa as ref

    def router(q, gk, lengths, scale):
        T = q.shape[2]
        reps = ref._completed_chunk_representatives(gk, chunk_size=64, valid_lengths=lengths,
                                                    representative_mode="mean_max_blend", blend_alpha=0.5)
        qn = F.normalize(q.float(), dim=-1, eps=1e-6).to(q.dtype)
        starts = torch.arange(-(-T // 16)) * 16
        anchor = qn[:, :, starts.clamp_max(T - 1)]
        logits = torch.matmul(anchor.float(), reps.float().transpose(-2, -1))
        meta = ref._build_causal_tile_metadata(anchor, gk, logits, chunk_size=64, top_k_chunks=4,
                                               top_m_tokens=64, selector_tile_size=16, valid_lengths=lengths,
                                               canonical_token_order=False, exploration_probability=0.0)
        route = ref._selected_route_scores(qn, reps, meta, scale)
        return reps, logits, meta, route

    # Router + lanes on raw Q/K/V: ragged length (5 chunks, last one partial),
    # per-row valid lengths, distinct local/global K/V.
    g = torch.Generator().manual_seed(21)
    B, H, T, D = 2, 2, 300, 64
    q = (torch.randn(B, H, T, D, generator=g) * 0.5).to(torch.bfloat16)
    lk = (torch.randn(B, H, T, D, generator=g) * 0.5).to(torch.bfloat16)
    lv = torch.randn(B, H, T, D, generator=g).to(torch.bfloat16)
    gk = (lk.float() + 0.3 * torch.randn(B, H, T, D, generator=g)).to(torch.bfloat16)
    gv = (lv.float() + 0.3 * torch.randn(B, H, T, D, generator=g)).to(torch.bfloat16)
    lengths = torch.tensor([300, 250], dtype=torch.int32)
    scale = torch.tensor([0.1, 0.35])
    reps, logits, meta, route = router(q, gk, lengths, scale)
    f32 = lambda t: t.float()
    lo, llse = ref._eager_local_lane(f32(q), f32(lk), f32(lv), lengths, local_window=64, selector_tile_size=16)
    go, glse = ref._eager_global_lane(f32(q), f32(gk), f32(gv), route.float(), meta, local_window=64)
    merged, mlse = ref._merge_attention_lanes(lo, llse, go, glse)
    save("hisa_router_lanes", q=q, local_key=lk, local_value=lv, global_key=gk, global_value=gv,
         valid_lengths=lengths, route_scale=scale, reps=reps, logits=logits, top_chunk_idx=meta.top_chunk_idx,
         route=route, merged=merged, merged_lse=mlse)

    # Router only, long enough that top-4 picks among up to 31 completed chunks.
    g = torch.Generator().manual_seed(22)
    B, H, T = 1, 4, 2048
    q = (torch.randn(B, H, T, D, generator=g) * 0.125).to(torch.bfloat16)
    gk = (torch.randn(B, H, T, D, generator=g) * 0.125).to(torch.bfloat16)
    lengths = torch.tensor([2048], dtype=torch.int32)
    reps, logits, meta, route = router(q, gk, lengths, torch.full((H,), 0.1))
    save("hisa_router_long", q=q, global_key=gk, valid_lengths=lengths, reps=reps, logits=logits,
         top_chunk_idx=meta.top_chunk_idx, route=route)

    # Whole module (eval, fp32, with an EMA/NPCI kv_inject packet), head_dim 64.
    module, x, kd, vd = _hisa_module_case(ref)
    with torch.no_grad():
        y = module(x, kv_inject=(kd, vd))
    state = {f"state.{k}": val for k, val in module.state_dict().items()}
    save("hisa_module_eval", x=x, key_delta=kd, value_delta=vd, y=y, **state)
    make_hisa_module_bf16()


def _hisa_module_case(ref):
    """The module-level HISA case: seeded module with non-trivial adapters, route prior and
    NPCI angles, a bf16-valued input and an fp32 kv_inject packet."""
    torch.manual_seed(4)
    module = ref.HierarchicalSparseAttentionV16HISACausal(
        D=128, H=2, hd=64, chunk_size=64, top_k_chunks=4, hisa_top_m_tokens=64, local_window=64,
        selector_tile_size=16, representative_mode="mean_max_blend", representative_blend_alpha=0.5,
        route_prior_scale=0.1, global_adapter_rank=16, npci_theta_max=0.25, local_backend="flex").eval()
    gen = torch.Generator().manual_seed(44)
    with torch.no_grad():
        for p in (module.global_k_up.weight, module.global_v_up.weight):
            p.copy_(torch.randn(p.shape, generator=gen) * 0.05)
        module.route_prior_raw.copy_(torch.tensor([-1.0, 0.5]))
        module.npci_theta_k.copy_(torch.tensor([1.5, -0.7]))
        module.npci_theta_v.copy_(torch.tensor([0.4, 2.0]))
    x = torch.randn(2, 200, 128, generator=gen).to(torch.bfloat16).float()
    kd = torch.randn(2, 2, 200, 64, generator=gen) * 0.5
    vd = torch.randn(2, 2, 200, 64, generator=gen) * 0.5
    return module, x, kd, vd


def make_hisa_module_bf16() -> None:
    """The module-level HISA case run by the reference in bf16 (module.to(bfloat16), bf16
    input and packet), the precision the engine computes in: hisa_module_eval_bf16."""
    _import_reference()
    import hierarchical_sparse_attn_v18_hisa as ref

    module, x, kd, vd = _hisa_module_case(ref)
    module = module.to(torch.bfloat16)
    with torch.no_grad():
        y = module(x.to(torch.bfloat16), kv_inject=(kd.to(torch.bfloat16), vd.to(torch.bfloat16)))
        _, meta = module(x.to(torch.bfloat16), kv_inject=(kd.to(torch.bfloat16), vd.to(torch.bfloat16)),
                         return_metadata=True)
    save("hisa_module_eval_bf16", y=y, top_chunk_idx=meta.top_chunk_idx, token_idx=meta.token_idx,
         token_scores=meta.token_scores, enumerate_all=np.asarray(meta.enumerate_all))


def make_hisa_backward() -> None:
    """Backward golden vectors: fp64 autograd through the reference's own eager
    lanes and merge (_eager_local_lane, _eager_global_lane, _merge_attention_lanes,
    hierarchical_sparse_attn_v18_hisa.py:688-835) on the committed router/lanes
    inputs, route a differentiable input, metadata from the reference router."""
    _import_reference()
    import hierarchical_sparse_attn_v18_hisa as ref

    sys.path.insert(0, str(HERE.parent.parent))
    from tests._golden import load

    g = load("hisa_router_lanes")
    T = g["q"].shape[2]
    meta = ref.HISAMetadata(top_chunk_idx=g["top_chunk_idx"], token_idx=torch.empty(0, dtype=torch.int32),
                            token_scores=torch.empty(0), tile_starts=torch.arange(-(-T // 16), dtype=torch.int32) * 16,
                            valid_lengths=g["valid_lengths"], chunk_size=64, selector_tile_size=16,
                            enumerate_all=True)
    names = ("q", "local_key", "local_value", "global_key", "global_value", "route")
    leaves = {n: g[n].double().clone().requires_grad_(True) for n in names}
    lo, llse = ref._eager_local_lane(leaves["q"], leaves["local_key"], leaves["local_value"], g["valid_lengths"],
                                     local_window=64, selector_tile_size=16)
    go, glse = ref._eager_global_lane(leaves["q"], leaves["global_key"], leaves["global_value"], leaves["route"],
                                      meta, local_window=64)
    merged, _ = ref._merge_attention_lanes(lo, llse, go, glse)
    dout = torch.randn(merged.shape, generator=torch.Generator().manual_seed(51), dtype=torch.float64)
    dout = dout.to(torch.bfloat16)
    grads = torch.autograd.grad(merged, [leaves[n] for n in names], dout.double())
    # Router auxiliary loss on the same inputs (every candidate tile, so no draw).
    import torch.nn.functional as F
    qn = F.normalize(g["q"].float(), dim=-1, eps=1e-6).to(g["q"].dtype)
    anchor = qn[:, :, (torch.arange(-(-T // 16)) * 16).clamp_max(T - 1)]
    logits = torch.matmul(anchor.float(), g["reps"].float().transpose(-2, -1))
    aux = ref._router_auxiliary_loss(logits, anchor, g["global_key"], meta, samples=64, temperature=1.0)
    # The random training paths under fixed CPU seeds: the auxiliary loss over 4
    # sampled tiles (torch.randperm) and the exploration slot (two torch.rand draws).
    torch.manual_seed(123)
    aux_sampled = ref._router_auxiliary_loss(logits, anchor, g["global_key"], meta, samples=4, temperature=1.0)
    tiles = -(-T // 16)
    eligible = ref._eligibility(torch.arange(tiles, dtype=torch.int32) * 16, g["reps"].shape[2], 64,
                                g["valid_lengths"])
    top3 = g["top_chunk_idx"][..., :3].contiguous()
    torch.manual_seed(124)
    explored, _ = ref._inject_exploration_slot(top3.long(), top3 >= 0, eligible, 0.5)
    save("hisa_bwd_lanes", dout=dout, merged=merged.detach().float(),
         **{f"d_{n}": gr.float() for n, gr in zip(names, grads)}, aux=aux, aux_sampled=aux_sampled,
         explored=explored.to(torch.int32))


def make_hisa_module_grad() -> None:
    """Training-mode gradients of the reference HISA module (CPU, fp32, exploration
    off, the router auxiliary loss over every candidate tile so that no tile is drawn
    at random): output, auxiliary loss, dx and every parameter's gradient of
    sum(y * dy) + aux, with and without a kv_inject packet. T=300 (the last chunk
    partial) with valid lengths 300 / 250; at most four chunks are eligible, so the
    routed set does not hinge on near-ties of the anchor logits."""
    _import_reference()
    import hierarchical_sparse_attn_v18_hisa as ref

    torch.manual_seed(5)
    module = ref.HierarchicalSparseAttentionV16HISACausal(
        D=128, H=2, hd=64, chunk_size=64, top_k_chunks=4, hisa_top_m_tokens=64, local_window=64,
        selector_tile_size=16, representative_mode="mean_max_blend", representative_blend_alpha=0.5,
        route_prior_scale=0.1, route_aux_weight=0.01, route_aux_samples=64, route_aux_temperature=1.0,
        exploration_probability=0.0, global_adapter_rank=16, npci_theta_max=0.25, local_backend="flex").train()
    gen = torch.Generator().manual_seed(55)
    with torch.no_grad():
        module.qkvg_proj.weight.mul_(4.0)
        for p in (module.global_k_up.weight, module.global_v_up.weight):
            p.copy_(torch.randn(p.shape, generator=gen) * 0.05)
        module.route_prior_raw.copy_(torch.tensor([-1.0, 0.5]))
        module.npci_theta_k.copy_(torch.tensor([1.5, -0.7]))
        module.npci_theta_v.copy_(torch.tensor([0.4, 2.0]))
    B, T = 2, 300
    x = torch.randn(B, T, 128, generator=gen).to(torch.bfloat16).float()
    kd = torch.randn(B, 2, T, 64, generator=gen) * 0.5
    vd = torch.randn(B, 2, T, 64, generator=gen) * 0.5
    dy = torch.randn(B, T, 128, generator=gen)
    lengths = torch.tensor([300, 250], dtype=torch.int32)
    state = {f"state.{k}": val for k, val in module.state_dict().items()}

    # A second run with the attention lanes fed and read at the bf16 points of a
    # bf16 attention kernel (q, K/V and the route prior rounded on the way in,
    # the merged output rounded on the way out, its incoming gradient rounded to
    # bf16; gradients to the inputs pass straight through): the reference's
    # fp32 maths otherwise unchanged.
    class _Round(torch.autograd.Function):
        @staticmethod
        def forward(ctx, t, round_grad):
            ctx.round_grad = round_grad
            return t.to(torch.bfloat16).to(t.dtype)

        @staticmethod
        def backward(ctx, grad):
            return (grad.to(torch.bfloat16).to(grad.dtype) if ctx.round_grad else grad), None

    local_lane, global_lane, merge = module._local_lane, ref._eager_global_lane, ref._merge_attention_lanes

    def bf16_local(q, k, v, lengths_):
        return local_lane(*(_Round.apply(t, False) for t in (q, k, v)), lengths_)

    def bf16_global(q, k, v, route, meta, **kw):
        return global_lane(*(_Round.apply(t, False) for t in (q, k, v, route)), meta, **kw)

    def bf16_merge(*args):
        merged, lse = merge(*args)
        return _Round.apply(merged, True), lse

    out = {}
    for points in ("", "bf16."):
        if points:
            module._local_lane = bf16_local
            ref._eager_global_lane, ref._merge_attention_lanes = bf16_global, bf16_merge
        for tag, inject in (("plain", None), ("inject", (kd, vd))):
            module.zero_grad()
            xl = x.clone().requires_grad_(True)
            y, aux = module(xl, kv_inject=inject, valid_lengths=lengths, return_auxiliary=True)
            ((y * dy).sum() + aux).backward()
            out[f"{points}{tag}.y"] = y.detach()
            out[f"{points}{tag}.aux"] = aux.detach()
            out[f"{points}{tag}.dx"] = xl.grad
            for name, p in module.named_parameters():
                if p.grad is not None:
                    out[f"{points}{tag}.grad.{name}"] = p.grad.clone()
    module._local_lane = local_lane
    ref._eager_global_lane, ref._merge_attention_lanes = global_lane, merge
    save("hisa_module_grad", x=x, kd=kd, vd=vd, dy=dy, valid_lengths=lengths, **state, **out)


def make_model_train() -> None:
    """One training step of the reference DwarfForCausalLM (small config: vocab 1024,
    D=128, H=2, FFN 384, T=256, B=2; seeded init; train mode, dropout 0, HISA
    exploration off and its auxiliary loss over every candidate tile, so the step
    has no random draws): loss = cross entropy of the next token + auxiliary loss.
    Run in fp32 (gradients stored rounded to bf16, loss, aux, logits at a few
    positions) and in bf16 (its per-parameter cosine and relative norm shift
    against the fp32 run, the spread that bf16 arithmetic alone causes)."""
    _import_reference()
    import train_dwarf as td

    cfg = td.DwarfConfig(vocab_size=1024, embedding_dim=128, num_heads=2, ffn_dim=384, seq_len=257, dropout=0.0)
    ids = torch.randint(57, 1024, (2, 256), generator=torch.Generator().manual_seed(0))
    positions = torch.tensor([0, 17, 100, 255])
    runs = {}
    for dtype in (torch.float32, torch.bfloat16):
        model = td.DwarfForCausalLM(cfg).to(dtype).train()
        for module in model.modules():
            if hasattr(module, "exploration_probability"):
                module.exploration_probability = 0.0
                module.route_aux_samples = 64
        logits, aux = model(ids, return_auxiliary=True)
        ce = F.cross_entropy(logits.reshape(-1, cfg.vocab_size).float(), ids.roll(-1, 1).reshape(-1))
        (ce + aux).backward()
        runs[dtype] = (logits.detach().float(), ce.detach(), aux.detach(),
                       {n: p.grad.detach().double() for n, p in model.named_parameters() if p.grad is not None})
    logits, ce, aux, grads = runs[torch.float32]
    _, ce16, aux16, grads16 = runs[torch.bfloat16]
    out = {"input_ids": ids, "positions": positions, "logits": logits[:, positions], "ce": ce, "aux": aux,
           "ce_bf16": ce16, "aux_bf16": aux16}
    for name, g32 in grads.items():
        g16 = grads16[name]
        out["grad." + name] = g32.to(torch.bfloat16)
        norm = float(g32.norm())
        out["cos_bf16." + name] = torch.tensor(float((g32 * g16).sum()) / max(norm * float(g16.norm()), 1e-30))
        out["norm_shift_bf16." + name] = torch.tensor(abs(float(g16.norm()) - norm) / max(norm, 1e-30))
    save("model_train_step", **out)


def make_hisa_backward_edges() -> None:
    """HISA attention backward at the edges, each case from the reference's own
    router (representatives, anchor logits, top-4) and fp64 autograd through its
    eager lanes + merge: T=64 (one chunk, so no tile has a routed chunk),
    T=1 (row 0 has no key), T=83 with valid lengths [83, 0] (a row of length 0
    and a partial last tile), T=200 with lengths [130, 199]."""
    _import_reference()
    import torch.nn.functional as F

    import hierarchical_sparse_attn_v18_hisa as ref

    out = {}
    cases = [("t64", 64, [64, 64]), ("t1", 1, [1, 1]), ("t83", 83, [83, 0]), ("t200", 200, [130, 199])]
    for i, (tag, T, lens) in enumerate(cases):
        g = torch.Generator().manual_seed(700 + i)
        B, H, D = 2, 2, 64
        q = (torch.randn(B, H, T, D, generator=g) * 0.5).to(torch.bfloat16)
        lk = (torch.randn(B, H, T, D, generator=g) * 0.5).to(torch.bfloat16)
        lv = torch.randn(B, H, T, D, generator=g).to(torch.bfloat16)
        gk = (lk.float() + 0.3 * torch.randn(B, H, T, D, generator=g)).to(torch.bfloat16)
        gv = (lv.float() + 0.3 * torch.randn(B, H, T, D, generator=g)).to(torch.bfloat16)
        lengths = torch.tensor(lens, dtype=torch.int32)
        reps = ref._completed_chunk_representatives(gk, chunk_size=64, valid_lengths=lengths,
                                                    representative_mode="mean_max_blend", blend_alpha=0.5)
        qn = F.normalize(q.float(), dim=-1, eps=1e-6).to(q.dtype)
        anchor = qn[:, :, (torch.arange(-(-T // 16)) * 16).clamp_max(T - 1)]
        logits = torch.matmul(anchor.float(), reps.float().transpose(-2, -1))
        meta = ref._build_causal_tile_metadata(anchor, gk, logits, chunk_size=64, top_k_chunks=4, top_m_tokens=64,
                                               selector_tile_size=16, valid_lengths=lengths,
                                               canonical_token_order=False, exploration_probability=0.0)
        route = ref._selected_route_scores(qn, reps, meta, torch.tensor([0.1, 0.3]))
        names = ("q", "local_key", "local_value", "global_key", "global_value", "route")
        leaves = {n: t.double().clone().requires_grad_(True) for n, t in zip(names, (q, lk, lv, gk, gv, route))}
        lo, llse = ref._eager_local_lane(leaves["q"], leaves["local_key"], leaves["local_value"], lengths,
                                         local_window=64, selector_tile_size=16)
        go, glse = ref._eager_global_lane(leaves["q"], leaves["global_key"], leaves["global_value"],
                                          leaves["route"], meta, local_window=64)
        merged, _ = ref._merge_attention_lanes(lo, llse, go, glse)
        dout = torch.randn(merged.shape, generator=g, dtype=torch.float64).to(torch.bfloat16)
        grads = torch.autograd.grad(merged, [leaves[n] for n in names], dout.double(), allow_unused=True)
        out.update({f"{tag}.{n}": t for n, t in zip(names, (q, lk, lv, gk, gv, route))})
        out[f"{tag}.valid_lengths"] = lengths
        out[f"{tag}.top_chunk_idx"] = meta.top_chunk_idx
        out[f"{tag}.dout"] = dout
        out[f"{tag}.merged"] = merged.detach().float()
        for n, gr in zip(names, grads):
            out[f"{tag}.d_{n}"] = (torch.zeros_like(leaves[n]) if gr is None else gr).float()
    save("hisa_bwd_edges", **out)


def make_model() -> None:
    """Whole-model prefill of the reference DwarfForCausalLM (seeded init), B=1, T=2048.

    bf16 weights/activations on CPU (the BASELINE config-5 precision), plus the
    same model in fp32, plus a q6 variant where every DSQG layer sees K/V
    round-tripped through the q6 codec (oracle/q6.py), z_pre from unquantised K.
    Stored: final hidden states at every 4th position, logits at 4 positions
    and a parameter digest.
    """
    import hashlib

    _import_reference()
    sys.path.insert(0, str(HERE.parent.parent))
    import dsqg_attention_v22 as ref_dsqg
    import train_dwarf as td

    from oracle import q6 as oq6

    model = td.DwarfForCausalLM(td.DwarfConfig()).eval()
    digest = hashlib.sha256()
    for name, tensor in model.state_dict().items():
        digest.update(name.encode())
        digest.update(tensor.detach().float().numpy().tobytes())
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(57, 32768, (1, 2048), generator=g)
    positions = torch.tensor([1, 65, 1024, 2047])       # logits kept at these positions
    rows = torch.arange(0, 2048, 4)                        # hidden states kept at these positions
    out = {"input_ids": ids, "positions": positions, "rows": rows,
           "param_count": sum(p.numel() for p in model.parameters()),
           "param_sha256": np.frombuffer(digest.digest(), dtype=np.uint8)}
    with torch.no_grad():
        h32 = model(ids, return_hidden=True)
        out["logits_f32"] = model.lm_head(h32)[0, positions]
        m16 = model.to(torch.bfloat16)
        h16 = m16(ids, return_hidden=True)
        out["hidden_bf16"] = h16[0, rows]
        out["logits_bf16"] = m16.lm_head(h16)[0, positions].float()
        original = ref_dsqg.dsqg_attention_v18_grouped

        def fake_q6(q, k, v, *args, **kwargs):
            def rt(t):
                codes, scales = oq6.pack(t.float().numpy())
                return torch.from_numpy(oq6.unpack(codes, scales)).to(t.dtype)
            return original(q, rt(k), rt(v), *args, **kwargs)

        ref_dsqg.dsqg_attention_v18_grouped = fake_q6
        try:
            hq = m16(ids, return_hidden=True)
        finally:
            ref_dsqg.dsqg_attention_v18_grouped = original
        out["hidden_bf16_q6"] = hq[0, rows]
        out["logits_bf16_q6"] = m16.lm_head(hq)[0, positions].float()
    save("model_prefill_b1_t2048", **out)


BLOCK_ROWS = slice(15, 2048, 16)  # output rows kept per block (128 rows, the last row included)


def make_model_blocks() -> None:
    """Per-block parity fixtures of the reference DwarfForCausalLM (seeded init), B=1, T=2048.

    Each of the 10 blocks (train/train_dwarf.py:320-322 DSQG, :356-364 HISA) runs
    on its own seeded input, randn(seed 100 + i) times the RMS of the block's real
    input in the reference bf16 prefill of the model_prefill token ids (the
    residual stream grows from 0.02 to ~0.3 over the blocks), cast to bf16.
    Stored per block, at rows BLOCK_ROWS: the bf16 model's block output, the fp32
    model's block output on the same (bf16-valued) input, and the bf16 model's
    block output with q6 round-tripped K/V in its DSQG attention (oracle/q6.py;
    DSQG blocks only). The inputs are regenerated by the test from the stored
    RMS, so the fixture stays small.
    """
    _import_reference()
    sys.path.insert(0, str(HERE.parent.parent))
    import dsqg_attention_v22 as ref_dsqg
    import train_dwarf as td

    from oracle import q6 as oq6

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    m32 = td.DwarfForCausalLM(td.DwarfConfig()).eval()
    m16 = td.DwarfForCausalLM(td.DwarfConfig()).eval().to(torch.bfloat16)
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(57, 32768, (1, 2048), generator=g)
    out = {"rows": torch.arange(2048)[BLOCK_ROWS]}
    original = ref_dsqg.dsqg_attention_v18_grouped

    def fake_q6(q, k, v, *args, **kwargs):
        def rt(t):
            codes, scales = oq6.pack(t.float().numpy())
            return torch.from_numpy(oq6.unpack(codes, scales)).to(t.dtype)
        return original(q, rt(k), rt(v), *args, **kwargs)

    def run(block, x):
        y = block(x)
        return y[0] if isinstance(y, tuple) else y

    with torch.no_grad():
        x = m16.embedding(ids)
        rms = []
        for block in m16.blocks:
            rms.append(float(x.float().square().mean().sqrt()))
            x = run(block, x)
        out["input_rms"] = torch.tensor(rms, dtype=torch.float64)
        for i, (b16, b32) in enumerate(zip(m16.blocks, m32.blocks)):
            xin = (torch.randn(1, 2048, 512, generator=torch.Generator().manual_seed(100 + i)) * rms[i])
            xin = xin.to(torch.bfloat16)
            out[f"block{i}_bf16"] = run(b16, xin)[0, BLOCK_ROWS]
            out[f"block{i}_f32"] = run(b32, xin.float())[0, BLOCK_ROWS]
            if not isinstance(b16, td.GlobalMixerBlock):
                ref_dsqg.dsqg_attention_v18_grouped = fake_q6
                try:
                    out[f"block{i}_bf16_q6"] = run(b16, xin)[0, BLOCK_ROWS]
                finally:
                    ref_dsqg.dsqg_attention_v18_grouped = original
    save("model_blocks_b1_t2048", **out)


def make_checkpoint() -> None:
    """Legacy-key migration of the reference modules' _load_from_state_dict.

    DSQG (dsqg_attention_v22.py:3069-3142): a V19/V20-style dict with separate
    qkv_proj / gate_proj (+ an out_proj.bias and the old unconstrained pos_bias
    table). HISA (hierarchical_sparse_attn_v18_hisa.py:2469-2544): separate
    W_q / W_k / W_v with the block-level gate_proj, and no adapter / NPCI /
    route-prior parameters. Stored: the legacy dict and the state the
    reference module holds after loading it.
    """
    _import_reference()
    import dsqg_attention_v22 as ref_dsqg
    import hierarchical_sparse_attn_v18_hisa as ref_hisa

    torch.manual_seed(5)
    offsets = [1, 2, 3, 5, 8, 13, 21, 48, 64, 100]
    src = ref_dsqg.DSQGAttentionV19(128, 2, offsets, 7, 3, seq_len=160, dropout=0.0, plane_shift=6)
    _randomize_dsqg(src, 505)
    sd = src.state_dict()
    D = 128
    legacy = {k: v.clone() for k, v in sd.items()
              if not k.startswith(("qkvg_proj.", "pos_bias_log_slope", "pos_bias_residual", "pos_bias_scale"))}
    legacy["qkv_proj.weight"] = sd["qkvg_proj.weight"][: 3 * D].clone()
    legacy["qkv_proj.bias"] = sd["qkvg_proj.bias"][: 3 * D].clone()
    legacy["gate_proj.weight"] = sd["qkvg_proj.weight"][3 * D:].clone()
    legacy["gate_proj.bias"] = sd["qkvg_proj.bias"][3 * D:].clone()
    legacy["out_proj.bias"] = torch.randn(D)
    legacy["pos_bias"] = torch.randn(len(offsets), 2) * 0.5
    torch.manual_seed(6)
    dst = ref_dsqg.DSQGAttentionV19(128, 2, offsets, 7, 3, seq_len=160, dropout=0.0, plane_shift=6)
    dst.load_state_dict({k: v.clone() for k, v in legacy.items()}, strict=True)
    out = {f"legacy.{k}": v for k, v in legacy.items()}
    out.update({f"loaded.{k}": v for k, v in dst.state_dict().items()})
    save("checkpoint_dsqg_legacy", **out)

    torch.manual_seed(7)
    kwargs = dict(D=128, H=2, hd=64, chunk_size=64, top_k_chunks=4, hisa_top_m_tokens=64, local_window=64,
                  selector_tile_size=16, representative_mode="mean_max_blend", representative_blend_alpha=0.5,
                  route_prior_scale=0.1, global_adapter_rank=16, npci_theta_max=0.25, local_backend="flex")
    src = ref_hisa.HierarchicalSparseAttentionV16HISACausal(**kwargs)
    sd = src.state_dict()
    gen = torch.Generator().manual_seed(77)
    legacy = {}
    for name in ("W_q", "W_k", "W_v"):
        legacy[f"attn.{name}.weight"] = torch.randn(D, D, generator=gen) * 0.05
        legacy[f"attn.{name}.bias"] = torch.randn(D, generator=gen) * 0.05
    legacy["gate_proj.weight"] = torch.randn(D, D, generator=gen) * 0.05
    legacy["gate_proj.bias"] = torch.randn(D, generator=gen) * 0.05
    for k, v in sd.items():
        if k.startswith(("qkvg_proj.", "route_prior_raw", "npci_theta_", "global_k_", "global_v_")):
            continue
        legacy[f"attn.{k}"] = v.clone()
    torch.manual_seed(8)
    dst = ref_hisa.HierarchicalSparseAttentionV16HISACausal(**kwargs)
    block = torch.nn.Module()  # stands in for the block that owns the legacy gate_proj
    block.attn = dst
    # strict=False: the stand-in block has no module of its own for the legacy gate keys
    result = block.load_state_dict({k: v.clone() for k, v in legacy.items()}, strict=False)
    assert not result.missing_keys, result
    out = {f"legacy.{k}": v for k, v in legacy.items()}
    out.update({f"loaded.{k}": v for k, v in dst.state_dict().items()})
    save("checkpoint_hisa_legacy", **out)


def main(argv: list[str]) -> None:
    which = argv[1] if len(argv) > 1 else "all"
    makers = {"ema": make_ema, "ema_bwd": make_ema_backward, "dsqg": make_dsqg, "dsqg_bwd": make_dsqg_backward, "dsqg_module_grad": make_dsqg_module_grad, "hisa": make_hisa, "hisa_module_bf16": make_hisa_module_bf16, "hisa_bwd": make_hisa_backward, "hisa_bwd_edges": make_hisa_backward_edges, "hisa_module_grad": make_hisa_module_grad, "model": make_model, "model_blocks": make_model_blocks, "model_train": make_model_train,
              "checkpoint": make_checkpoint}
    for name, maker in makers.items():
        if which in ("all", name):
            maker()


if __name__ == "__main__":
    main(sys.argv)
