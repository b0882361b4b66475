"""Per-kernel measurements at the benchmark configuration shapes.

``python -m dwarf_v2_b200.kernel_bench [--case NAME ...] [--iters K] [--warmup W]``
prints one JSON line per case: the mean device time of each engine entry point
the case launches (CUDA events around every launch on the launching stream,
``_lib.LaunchLog``), the algorithmic bytes (and FLOPs where they matter) of the
case's main kernel, and the achieved rate against the measured HBM peak in
``MEASURED_PEAKS.json`` (repository root) or, when that file is absent, the
pool's earlier measurement (6650 GB/s, marked "fallback").

Inputs are synthetic, seeded, with the shapes and distributions of the named
configurations (config 2: causal EMA scan B=16 T=2048 D=512 fp32; config 3:
DSQG over a q6 KV cache B=32 H=8 T=2048 J=96; config 4: HISA B=32 H=8 T=2048,
Q/K/V ~ N(0, 0.125^2)); the backward cases use the same shapes; the training
step case runs the full model on 8 x 2048 tokens. Before every timed iteration
a 512 MB buffer is written, so no input starts in the 126 MB L2.
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch

from . import _lib

FALLBACK_HBM_GBS = 6650.0


def _hbm_peak() -> tuple[float, str]:
    path = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    if path.is_file():
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def _nbytes(*tensors: torch.Tensor) -> int:
    return sum(t.numel() * t.element_size() for t in tensors)


class _Timer:
    """Runs ``fn`` ``warmup`` times untimed, then ``iters`` times with an L2 flush before
    each and every engine launch timed with CUDA events."""

    def __init__(self, warmup: int, iters: int):
        self.warmup, self.iters = warmup, iters
        self.flush = torch.empty(512 << 20, dtype=torch.uint8, device="cuda")

    def __call__(self, fn, names: tuple[str, ...]) -> dict[str, float]:
        for _ in range(self.warmup):
            fn()
        torch.cuda.synchronize()
        log = _lib.LaunchLog(timed=names)
        for _ in range(self.iters):
            self.flush.fill_(1)
            _lib.set_launch_log(log)
            try:
                fn()
            finally:
                _lib.set_launch_log(None)
        torch.cuda.synchronize()
        return {n: log.mean_ms(n) for n in names if log.mean_ms(n) is not None}


def _rate(nbytes: int, ms: float, peak: float) -> dict:
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"algorithmic_bytes": nbytes, "achieved_gbs": round(gbs, 1), "frac_of_hbm_peak": round(gbs / peak, 4)}


def case_ema_config2(timer, peak):
    """Config 2: per-channel EMA scan, fp32 [16, 2048, 512] -> fp32."""
    from .causal_ema_scan import causal_ema_scan_per_channel

    g = torch.Generator().manual_seed(0)
    x = torch.randn(16, 2048, 512, generator=g).cuda()
    alpha = (1.0 - torch.sigmoid(torch.randn(512, generator=g))).cuda()
    out = {}
    times = timer(lambda: out.__setitem__("y", causal_ema_scan_per_channel(x, alpha)), ("dwarf_ema_scan",))
    ms = times["dwarf_ema_scan"]
    return {"kernel": "dwarf_ema_scan", "ms": ms, **_rate(2 * _nbytes(x), ms, peak)}


def case_ema_model_bf16(timer, peak):
    """The model's packet scans: scalar alpha, bf16 [32, 2048, 512] (32 rows = one GPU's
    share of the 256-row prefill batch at 8 GPUs)."""
    from .causal_ema_scan import causal_ema_scan

    g = torch.Generator().manual_seed(1)
    x = torch.randn(32, 2048, 512, generator=g).to(torch.bfloat16).cuda()
    alpha = torch.tensor([1.0 / 16.0], device="cuda")
    times = timer(lambda: causal_ema_scan(x, alpha), ("dwarf_ema_scan",))
    ms = times["dwarf_ema_scan"]
    return {"kernel": "dwarf_ema_scan", "ms": ms, **_rate(2 * _nbytes(x), ms, peak)}


def case_copy_config2(timer, peak):
    """Reference point, not an engine kernel: a device-to-device copy of the config-2 tensor
    (fp32 [16, 2048, 512], 67 MB read + 67 MB written, the EMA scan's bytes), timed with
    CUDA events after the same L2 flush: what a plain stream of this size reaches here."""
    g = torch.Generator().manual_seed(0)
    x = torch.randn(16, 2048, 512, generator=g).cuda()
    y = torch.empty_like(x)
    for _ in range(timer.warmup):
        y.copy_(x)
    times = []
    for _ in range(timer.iters):
        timer.flush.fill_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        y.copy_(x)
        b.record()
        times.append((a, b))
    torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in times) / len(times)
    return {"kernel": "torch copy_ (reference point)", "ms": ms, **_rate(2 * _nbytes(x), ms, peak)}


def case_ema_model_bf16_b256(timer, peak):
    """The packet scans of the config-5 prefill on one GPU: scalar alpha, bf16 [256, 2048, 512]."""
    from .causal_ema_scan import causal_ema_scan

    g = torch.Generator().manual_seed(1)
    x = torch.randn(256, 2048, 512, generator=g).to(torch.bfloat16).cuda()
    alpha = torch.tensor([1.0 / 16.0], device="cuda")
    times = timer(lambda: causal_ema_scan(x, alpha), ("dwarf_ema_scan",))
    ms = times["dwarf_ema_scan"]
    return {"kernel": "dwarf_ema_scan", "ms": ms, **_rate(2 * _nbytes(x), ms, peak)}


def case_ema_bwd_config2(timer, peak):
    """Config-2 backward: dx (the scan over time-reversed dy) and d alpha (one pass over
    x, y and dx)."""
    from .causal_ema_scan import causal_ema_scan_per_channel

    g = torch.Generator().manual_seed(2)
    x = torch.randn(16, 2048, 512, generator=g).cuda().requires_grad_(True)
    alpha = (1.0 - torch.sigmoid(torch.randn(512, generator=g))).cuda().requires_grad_(True)
    dy = torch.randn(16, 2048, 512, generator=g).cuda()
    y = causal_ema_scan_per_channel(x, alpha)

    def step():
        x.grad = alpha.grad = None
        torch.autograd.backward(y, dy, retain_graph=True)

    times = timer(step, ("dwarf_ema_scan", "dwarf_ema_scan_grad_alpha"))
    return {"kernels": times,
            "dwarf_ema_scan": _rate(2 * _nbytes(x), times["dwarf_ema_scan"], peak),
            "dwarf_ema_scan_grad_alpha": _rate(3 * _nbytes(x), times["dwarf_ema_scan_grad_alpha"], peak)}


def case_q6_pack_config3(timer, peak):
    """Config-3 K (or V) cache quantisation: bf16 [32, 8, 2048, 64] -> codes + fp16 scales."""
    from .q6 import q6_pack

    g = torch.Generator().manual_seed(3)
    k = torch.randn(32, 8, 2048, 64, generator=g).to(torch.bfloat16).cuda()
    res = {}
    times = timer(lambda: res.__setitem__("c", q6_pack(k)), ("dwarf_q6_pack",))
    codes, scales = res["c"]
    ms = times["dwarf_q6_pack"]
    return {"kernel": "dwarf_q6_pack", "ms": ms, **_rate(_nbytes(k, codes, scales), ms, peak)}


def case_q6_unpack_config3(timer, peak):
    """Config-3 K (or V) cache dequantisation: codes + fp16 scales -> bf16 [32, 8, 2048, 64]."""
    from .q6 import q6_pack, q6_unpack

    g = torch.Generator().manual_seed(3)
    codes, scales = q6_pack(torch.randn(32, 8, 2048, 64, generator=g).to(torch.bfloat16).cuda())
    res = {}
    times = timer(lambda: res.__setitem__("x", q6_unpack(codes, scales, torch.bfloat16)), ("dwarf_q6_unpack",))
    ms = times["dwarf_q6_unpack"]
    return {"kernel": "dwarf_q6_unpack", "ms": ms, **_rate(_nbytes(codes, scales, res["x"]), ms, peak)}


def case_packet_model_b256(timer, peak):
    """The InterferencePacket epilogue at the model's single-GPU shape: three bf16 scans and the
    gate pre-activation [256 x 2048, 512] -> the bf16 packet."""
    from .glue import packet

    g = torch.Generator(device="cuda").manual_seed(6)
    rows, width = 256 * 2048, 512
    scans = [torch.randn(rows, width, generator=g, device="cuda", dtype=torch.bfloat16) * s for s in (0.05, 0.1, 0.3)]
    gate_pre = torch.randn(rows, width, generator=g, device="cuda", dtype=torch.bfloat16)
    mixture = [0.33203125, 0.333984375, 0.333984375]
    res = {}
    times = timer(lambda: res.__setitem__("o", packet(scans, mixture, gate_pre)), ("dwarf_packet",))
    ms = times["dwarf_packet"]
    return {"kernel": "dwarf_packet", "ms": ms, **_rate(5 * _nbytes(gate_pre), ms, peak)}


def case_npci_model_b256(timer, peak):
    """The DSQG key rotation at the model's single-GPU shape (B=256, H=8, T=2048): key is the
    strided view of the fused qkvg projection, delta the strided view of the packet's kv output."""
    from .npci import npci_rotate_cuda

    g = torch.Generator(device="cuda").manual_seed(5)
    B, H, T = 256, 8, 2048
    qkvg = torch.randn(B, T, 4, H, 64, generator=g, device="cuda", dtype=torch.bfloat16)
    kv = torch.randn(B, T, 2, H, 64, generator=g, device="cuda", dtype=torch.bfloat16) * 0.3
    key, delta = qkvg[:, :, 1].permute(0, 2, 1, 3), kv[:, :, 0].permute(0, 2, 1, 3)
    theta = torch.full((H,), 0.2, device="cuda")
    out = torch.empty(B, H, T, 64, device="cuda", dtype=torch.bfloat16)
    times = timer(lambda: npci_rotate_cuda(key, delta, theta, out=out), ("dwarf_npci_rotate",))
    ms = times["dwarf_npci_rotate"]
    return {"kernel": "dwarf_npci_rotate", "ms": ms, **_rate(3 * _nbytes(out), ms, peak)}


def case_gemm_model_epilogues(timer, peak):
    """The model's fused-epilogue GEMMs (M = 128 x 2048 rows) beside the same GEMM with a
    plain store: qkvg + probes + q6 pack (N=2048, K=512), up_gate + SwiGLU (the model's
    hidden width padded to 1664: N=3328, K=512), down + residual + RMSNorm (N=512,
    K=1664), out_proj (N=512, K=512), lm_head (N=32768, K=512). FLOPs count the padded shapes the GEMMs run."""
    from . import gemm
    from .dsqg_attention_v22 import R_PLANES, _orthogonal_phase_probes

    g = torch.Generator(device="cuda").manual_seed(7)
    B, T, D, H = 128, 2048, 512, 8
    M = B * T

    def rnd(*shape, scale=1.0):
        return torch.randn(*shape, generator=g, device="cuda", dtype=torch.bfloat16) * scale

    x = rnd(B, T, D)
    out = {}
    qp, kp = (t.cuda() for t in _orthogonal_phase_probes(R_PLANES, 64))
    w_qkvg, b_qkvg = rnd(4 * D, D, scale=0.04), rnd(4 * D, scale=0.01)
    from .model import DwarfConfig, SwiGLUFFN

    ffn = SwiGLUFFN(DwarfConfig()).cuda()  # the model's own padded, interleaved FFN weights
    w_ug, w_down, tile = ffn._fused_weights()
    h = rnd(B, T, w_down.shape[1])
    w_out = rnd(D, D, scale=0.04)
    w_vocab = rnd(32768, D, scale=0.02)
    resid, nw = rnd(B, T, D), torch.ones(D, device="cuda")
    cases = {
        "qkvg_prep": (lambda: gemm.qkvg_prep(x, w_qkvg, b_qkvg, H, qp, kp), 2 * M * 4 * D * D),
        "qkvg_plain": (lambda: out.__setitem__("a", gemm.linear(x, w_qkvg, b_qkvg)), 2 * M * 4 * D * D),
        "up_gate_swiglu": (lambda: out.__setitem__("b", gemm.linear_swiglu(x, w_ug, tile)), 2 * M * w_ug.shape[0] * D),
        "up_gate_plain": (lambda: out.__setitem__("b", gemm.linear(x, w_ug)), 2 * M * w_ug.shape[0] * D),
        "down_rmsnorm": (lambda: gemm.linear_add_rmsnorm(h, w_down, resid, nw, x_out=resid),
                         2 * M * D * w_down.shape[1]),
        "down_plain": (lambda: out.__setitem__("c", gemm.linear(h, w_down)), 2 * M * D * w_down.shape[1]),
        "out_proj_plain": (lambda: out.__setitem__("d", gemm.linear(x, w_out)), 2 * M * D * D),
        "lm_head_plain": (lambda: out.__setitem__("e", gemm.linear(x, w_vocab)), 2 * M * 32768 * D),
    }
    res = {}
    for name, (fn, flops) in cases.items():
        ms = timer(fn, ("dwarf_gemm_bf16",))["dwarf_gemm_bf16"]
        res[name] = {"ms": round(ms, 4), "tflops": round(flops / (ms * 1e-3) / 1e12, 1)}
        out.clear()
    return {"rows": M, "gemms": res}


def _dsqg_tables(J: int, js: int, H: int, offsets, g):
    pb = torch.randn(J, H, generator=g) * 0.3 - torch.log1p(torch.tensor(offsets, dtype=torch.float32))[:, None]
    return (pb.cuda(), (torch.randn(J, 64, generator=g) * 0.05).cuda(),
            (torch.randn(J - js, H, 4, generator=g) * 0.5).cuda(), (torch.randn(J - js, H, 4, generator=g) * 2.0).cuda())


def case_dsqg_q6_config3(timer, peak):
    """Config 3: DSQG over a q6 KV cache, B=32 H=8 T=2048, the full 96-offset lattice."""
    from .dsqg_attention_v22 import ALL_OFFSETS, dsqg_attention_q6
    from .q6 import q6_pack

    g = torch.Generator().manual_seed(4)
    B, H, N, J, js = 32, 8, 2048, len(ALL_OFFSETS), 17
    q = torch.randn(B, H, N, 64, generator=g).to(torch.bfloat16).cuda()
    kc, ks = q6_pack(torch.randn(B, H, N, 64, generator=g).to(torch.bfloat16).cuda())
    vc, vs = q6_pack(torch.randn(B, H, N, 64, generator=g).to(torch.bfloat16).cuda())
    pb, se, pbase, pgain = _dsqg_tables(J, js, H, ALL_OFFSETS, g)
    y = (torch.randn(B, H, N, 4, generator=g) * 0.2).cuda()
    z = (torch.randn(B, H, N, 4, generator=g) * 0.2).cuda()
    offs = torch.tensor(ALL_OFFSETS, dtype=torch.int32, device="cuda")
    res = {}
    times = timer(lambda: res.__setitem__("o", dsqg_attention_q6(q, kc, ks, vc, vs, pb, se, pbase, pgain, y, z,
                                                                  offs, js, J - js, 0, 1)), ("dwarf_dsqg_fwd",))
    ms = times["dwarf_dsqg_fwd"]
    valid_pairs = sum(max(0, N - d) for d in ALL_OFFSETS) * B * H
    flops = valid_pairs * 4 * 64  # q.k and p.v: 2 x 64 FMAs per (query, offset) pair
    return {"kernel": "dwarf_dsqg_fwd (q6, 96 offsets)", "ms": ms,
            **_rate(_nbytes(q, kc, ks, vc, vs, y, z, res["o"]), ms, peak),
            "valid_pairs": valid_pairs, "fp32_tflops": round(flops / (ms * 1e-3) / 1e12, 2)}


def case_dsqg_q6_model_group(timer, peak):
    """One model DSQG layer over a q6 KV cache at the config-3 shape (B=32 H=8 T=2048) with
    the model's first 29-offset group (6 small, 23 large), the q6 cache layout the qkvg
    epilogue writes."""
    from .dsqg_attention_v22 import dsqg_attention_q6
    from .model import DwarfConfig, build_offset_groups
    from .q6 import q6_pack

    offsets = list(build_offset_groups(DwarfConfig())[0])
    js = sum(1 for o in offsets if o <= 28)
    g = torch.Generator().manual_seed(10)
    B, H, N, J = 32, 8, 2048, len(offsets)
    q = torch.randn(B, H, N, 64, generator=g).to(torch.bfloat16).cuda()
    kc, ks = q6_pack(torch.randn(B, H, N, 64, generator=g).to(torch.bfloat16).cuda())
    vc, vs = q6_pack(torch.randn(B, H, N, 64, generator=g).to(torch.bfloat16).cuda())
    pb, se, pbase, pgain = _dsqg_tables(J, js, H, offsets, g)
    y = (torch.randn(B, H, N, 4, generator=g) * 0.2).cuda()
    z = (torch.randn(B, H, N, 4, generator=g) * 0.2).cuda()
    offs = torch.tensor(offsets, dtype=torch.int32, device="cuda")
    res = {}
    times = timer(lambda: res.__setitem__("o", dsqg_attention_q6(q, kc, ks, vc, vs, pb, se, pbase, pgain, y, z,
                                                                  offs, js, J - js, 0, 1)), ("dwarf_dsqg_fwd",))
    ms = times["dwarf_dsqg_fwd"]
    valid_pairs = sum(max(0, N - d) for d in offsets) * B * H
    return {"kernel": "dwarf_dsqg_fwd (q6, model group 0)", "ms": ms,
            **_rate(_nbytes(q, kc, ks, vc, vs, y, z, res["o"]), ms, peak), "valid_pairs": valid_pairs,
            "fp32_tflops": round(valid_pairs * 4 * 64 / (ms * 1e-3) / 1e12, 2),
            "ns_per_pair_per_sm": round(ms * 1e6 * 148 / valid_pairs, 3)}


def case_dsqg_bwd_model_group(timer, peak):
    """DSQG backward at the config-3 shape (B=32 H=8 T=2048) with bf16 K/V and the model's
    first 29-offset group (one training layer): query-side and key-side gather kernels."""
    from .dsqg_attention_v22 import ALL_OFFSETS, dsqg_attention_v18_grouped

    offsets = [o for o in sorted(ALL_OFFSETS) if 2048 - o >= 64][0::3]
    js = sum(1 for o in offsets if o <= 28)
    J = len(offsets)
    g = torch.Generator().manual_seed(5)
    B, H, N = 32, 8, 2048
    r = lambda *s, std=1.0: (torch.randn(*s, generator=g) * std).cuda()  # noqa: E731
    leaves = [r(B, H, N, 64).bfloat16(), r(B, H, N, 64).bfloat16(), r(B, H, N, 64).bfloat16(), r(J, H, std=0.3),
              r(J, 64, std=0.3), r(J - js, H, 4, std=0.7), r(J - js, H, 4, std=2.0),
              r(B, H, N, 4, std=0.5).clamp(-1, 1), r(B, H, N, 4, std=0.5).clamp(-1, 1)]
    for t in leaves:
        t.requires_grad_(True)
    dout = r(B, H, N, 64).bfloat16()
    offs = torch.tensor(offsets, dtype=torch.int32, device="cuda")
    e = torch.empty(0, dtype=torch.int32, device="cuda")

    def step():
        for t in leaves:
            t.grad = None
        out = dsqg_attention_v18_grouped(*leaves, J, js, J - js, offs, e, e, e, e, e, 3, 0, False, 0, 0, 0)
        out.backward(dout)

    times = timer(step, ("dwarf_dsqg_fwd", "dwarf_dsqg_bwd"))
    q = leaves[0]
    # per (b,h,t) row: q, k, v, O, dO read, dq, dk, dv written (bf16 in, fp32 gradients out)
    row_bytes = 5 * 128 + 3 * 256
    return {"kernels": times, "offsets": J,
            "dwarf_dsqg_bwd": _rate(row_bytes * B * H * N, times["dwarf_dsqg_bwd"], peak)}


def _hisa_inputs(seed: int):
    g = torch.Generator().manual_seed(seed)
    B, H, T = 32, 8, 2048
    return [(torch.randn(B, H, T, 64, generator=g) * 0.125).to(torch.bfloat16).cuda() for _ in range(3)]


def case_hisa_config4(timer, peak):
    """Config 4: HISA router + fused tile attention, B=32 H=8 T=2048, local = global K/V."""
    from .hierarchical_sparse_attn_v18_hisa import hisa_attention

    q, k, v = _hisa_inputs(6)
    scale = torch.full((8,), 0.1)
    res = {}
    names = ("dwarf_hisa_reps", "dwarf_hisa_select", "dwarf_hisa_route", "dwarf_hisa_attn")
    times = timer(lambda: res.__setitem__("r", hisa_attention(q, k, v, k, v, scale, want_route=True)), names)
    out, top, route = res["r"]
    ms = times["dwarf_hisa_attn"]
    B, H, T = q.shape[:3]
    tiles = -(-T // 16)
    keys = 80 + 4 * 64  # the tile's local window rows and four routed chunks
    flops = tiles * B * H * 16 * keys * 64 * 4
    return {"kernels": times, "dwarf_hisa_attn": {**_rate(_nbytes(q, k, v, out, route, top), ms, peak),
                                                  "dense_tile_tflops": round(flops / (ms * 1e-3) / 1e12, 1)}}


def case_hisa_bwd_config4(timer, peak):
    """HISA fused tile attention backward at the config-4 shape (distinct local and global
    K/V, route prior requiring grad)."""
    from .hierarchical_sparse_attn_v18_hisa import chunk_representatives, hisa_tile_attention, route_prior
    from .hierarchical_sparse_attn_v18_hisa import select_chunks

    q, lk, lv = _hisa_inputs(7)
    _, gk, gv = _hisa_inputs(8)
    B, H, T = q.shape[:3]
    lengths = torch.full((B,), T, dtype=torch.int32, device="cuda")
    reps = chunk_representatives(gk, lengths, blend_alpha=0.5)
    top, _ = select_chunks(q, reps, lengths, top_k=4, temperature=1.0)
    route = route_prior(q, reps, top, torch.full((H,), 0.1, device="cuda")).float()
    leaves = [t.clone().requires_grad_(True) for t in (q, lk, lv, gk, gv, route)]
    dout = torch.randn(B, H, T, 64, device="cuda").to(torch.bfloat16)

    def step():
        for t in leaves:
            t.grad = None
        out = hisa_tile_attention(*leaves, top)
        out.backward(dout)

    times = timer(step, ("dwarf_hisa_attn", "dwarf_hisa_attn_bwd"))
    # reads q, O, dO and each key row touched (k, v of the local window and routed chunks:
    # counted once per tensor), writes dq and the four K/V gradients in fp32 and d route
    nbytes = 7 * _nbytes(q) + 5 * 2 * _nbytes(q) + B * H * T * 4 * 4
    return {"kernels": times, "dwarf_hisa_attn_bwd": _rate(nbytes, times["dwarf_hisa_attn_bwd"], peak)}


def case_model_train_step(timer, peak):
    """One training step of the full model (DwarfConfig(): D=512, L=10, vocab 32768, bf16
    weights, train mode) on B=8 x T=2048 tokens: forward, next-token cross entropy + the
    HISA auxiliary loss, backward. Whole-step time with CUDA events; the engine kernels'
    per-launch times inside the step."""
    import torch.nn.functional as F

    from .model import DwarfConfig, DwarfForCausalLM

    model = DwarfForCausalLM(DwarfConfig()).to(torch.bfloat16).cuda().train()
    g = torch.Generator().manual_seed(9)
    B, T = 8, 2048
    ids = torch.randint(57, 32768, (B, T), generator=g).cuda()
    labels = ids.roll(-1, 1).reshape(-1)

    def step():
        model.zero_grad(set_to_none=True)
        logits, aux = model(ids, return_auxiliary=True)
        loss = F.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(), labels) + aux
        loss.backward()

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    iters = 3
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        step()
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / iters
    names = ("dwarf_dsqg_fwd", "dwarf_dsqg_bwd", "dwarf_hisa_attn", "dwarf_hisa_attn_bwd", "dwarf_ema_scan",
             "dwarf_ema_scan_grad_alpha")
    return {"tokens_per_step": B * T, "ms_per_step": round(ms, 3), "train_tok_per_s": round(B * T / (ms * 1e-3)),
            "kernels_mean_ms": timer(step, names)}


CASES = {
    "ema_config2": case_ema_config2,
    "ema_model_bf16": case_ema_model_bf16,
    "ema_model_bf16_b256": case_ema_model_bf16_b256,
    "copy_config2": case_copy_config2,
    "ema_bwd_config2": case_ema_bwd_config2,
    "q6_pack_config3": case_q6_pack_config3,
    "q6_unpack_config3": case_q6_unpack_config3,
    "npci_model_b256": case_npci_model_b256,
    "packet_model_b256": case_packet_model_b256,
    "gemm_model_epilogues": case_gemm_model_epilogues,
    "dsqg_q6_config3": case_dsqg_q6_config3,
    "dsqg_q6_model_group": case_dsqg_q6_model_group,
    "dsqg_bwd_model_group": case_dsqg_bwd_model_group,
    "hisa_config4": case_hisa_config4,
    "hisa_bwd_config4": case_hisa_bwd_config4,
    "model_train_step": case_model_train_step,
}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--case", action="append", choices=sorted(CASES), help="cases to run (default: all)")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("kernel_bench needs a CUDA device")
    peak, peak_kind = _hbm_peak()
    timer = _Timer(args.warmup, args.iters)
    for name in args.case or list(CASES):
        result = CASES[name](timer, peak)
        print(json.dumps({"case": name, **result, "hbm_peak_gbs": peak, "peak": peak_kind}), flush=True)
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
