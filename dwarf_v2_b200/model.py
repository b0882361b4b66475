"""DWARF-v2 model construction API and whole-model prefill on B200.

Mirrors the model part of the reference trainer (train/train_dwarf.py:115-470):
``DwarfConfig``, ``build_offset_groups``, ``RMSNorm``, ``SwiGLUFFN``,
``InterferencePacket``, ``DSQGBlock``, ``GlobalMixerBlock`` and
``DwarfForCausalLM`` with the same module tree, parameter names and shapes
(55,348,728 parameters, 55,344,120 trainable) and the same seeded
initialisation (``reset_parameters``), so reference state dicts load unchanged
and a freshly built model holds bit-identical weights.

``DwarfForCausalLM.forward`` runs the prefill through this engine's kernels:
embedding + RMSNorm, per block the attention kernels, residual add fused with
the next RMSNorm (and, after the HISA block, with its sigmoid output gate),
SwiGLU, the EMA packet (three look-back scans + one epilogue kernel); every
GEMM runs on the engine's tcgen05 GEMM (``dwarf_gemm_bf16``, fused epilogues
for qkvg + DSQG prep, SwiGLU and residual + RMSNorm). Activations are bf16 with
the reference's rounding points.
``kv_cache="q6"`` runs every DSQG layer over the q6-quantised K/V cache.
Calls that need gradients (training mode, or autograd on with parameters that
require grad) take the reference's own block formulas as torch ops over the
engine's differentiable DSQG, HISA and EMA-scan functions (forward and backward
kernels); ``forward_lse`` and the decode entry points are inference-only.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Iterable

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib, gemm, glue
from .causal_ema_scan import bounded_ema_factor, causal_ema_scan, inverse_bounded_ema_factor
from .dsqg_attention_v22 import ALL_OFFSETS, R_PLANES, DSQGAttentionV19
from .hierarchical_sparse_attn_v18_hisa import HierarchicalSparseAttentionV16HISACausal, chunk_representatives

EXPECTED_PARAMETERS = 55_348_728
EXPECTED_TRAINABLE_PARAMETERS = 55_344_120
LAYOUT: tuple[int | None, ...] = (0, 1, 2, None, 0, 1, 2, 0, 1, 2)  # None = the HISA global mixer


@dataclass(frozen=True)
class DwarfConfig:
    """Model hyper-parameters (reference train/train_dwarf.py:115-151)."""

    vocab_size: int = 32768
    embedding_dim: int = 512
    num_heads: int = 8
    ffn_dim: int = 2400
    seq_len: int = 2048
    num_layers: int = 10
    dropout: float = 0.05
    min_offset_support: int = 64
    hisa_chunk_size: int = 64
    top_k_chunks: int = 4
    hisa_top_m_tokens: int = 64
    hisa_local_window: int = 64
    hisa_selector_tile: int = 16
    hisa_global_adapter_rank: int = 16
    ema_timescales: tuple[float, ...] = (16.0, 64.0, 256.0)
    init_seed: int = 42

    def __post_init__(self) -> None:
        if self.embedding_dim % self.num_heads:
            raise ValueError("embedding_dim must be divisible by num_heads")
        if self.num_layers != 10:
            raise ValueError("the 55M DWARF topology has exactly ten blocks")
        if self.seq_len < 65:
            raise ValueError("seq_len must be at least 65")
        head_dim = self.embedding_dim // self.num_heads
        if head_dim & (head_dim - 1):
            raise ValueError("HISA requires a power-of-two head dimension")

    @property
    def model_length(self) -> int:
        return self.seq_len - 1

    @property
    def swiglu_dim(self) -> int:
        return max(64, int(round((2.0 * self.ffn_dim / 3.0) / 64.0)) * 64)


def build_offset_groups(config: DwarfConfig) -> tuple[tuple[int, ...], ...]:
    """Offsets with >= min_offset_support sources at model length, dealt round-robin into 3 groups (reference :157-169)."""
    offsets = tuple(sorted(int(v) for v in ALL_OFFSETS))
    if len(offsets) != len(set(offsets)):
        raise ValueError("canonical DSQG offsets must be unique")
    live = tuple(d for d in offsets if config.model_length - d >= config.min_offset_support)
    groups = tuple(tuple(live[i::3]) for i in range(3))
    if any(not g for g in groups):
        raise ValueError("offset pruning left an empty DSQG group")
    return groups


def _small_large_counts(offsets: Iterable[int]) -> tuple[int, int]:
    values = tuple(int(v) for v in offsets)
    small = sum(v <= 28 for v in values)
    large = sum(v >= 48 for v in values)
    if small + large != len(values):
        raise ValueError("DSQG offsets must remain in the supported kernel bands")
    return small, large


def _act(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)


def _wants_grad(module: nn.Module, *tensors: torch.Tensor) -> bool:
    """True when a forward must be differentiable (or apply training-mode randomness):
    the module is training, or autograd is on and an input or a parameter requires grad.
    Such calls take the reference's own formulas as torch ops, with the engine's
    differentiable attention / scan functions; the rest take the fused inference kernels."""
    if module.training:
        return True
    if not torch.is_grad_enabled():
        return False
    return any(t.requires_grad for t in tensors) or any(p.requires_grad for p in module.parameters())


class RMSNorm(nn.Module):
    def __init__(self, dimension: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dimension))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if _wants_grad(self, x):  # reference train/train_dwarf.py:224-227
            xf = x.float()
            normalized = xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + self.eps)
            return (normalized * self.weight.float()).to(x.dtype)
        return glue.rmsnorm(_act(x), self.weight.detach(), self.eps)


class SwiGLUFFN(nn.Module):
    def __init__(self, config: DwarfConfig) -> None:
        super().__init__()
        hidden = config.swiglu_dim
        self.up_gate = nn.Linear(config.embedding_dim, 2 * hidden, bias=False)
        self.down = nn.Linear(hidden, config.embedding_dim, bias=False)
        self.dropout = nn.Dropout(config.dropout)

    def _fused_weights(self) -> tuple[torch.Tensor, torch.Tensor, int]:
        """Weights of the fused FFN GEMMs, cached per weight version.

        The hidden width is padded to a multiple of 128 with zero up/gate rows
        and zero down columns (silu(0) * 0 = 0 and zero columns add exact zeros,
        so results are unchanged), which lets the SwiGLU GEMM use 256-wide tiles
        (128 up + 128 gate columns); the up_gate rows are tile-interleaved."""
        w, wd = self.up_gate.weight, self.down.weight
        key = (w.data_ptr(), w._version, wd.data_ptr(), wd._version, w.device)
        if getattr(self, "_fw_key", None) != key:
            hidden = w.shape[0] // 2
            tile = 128
            padded = -(-hidden // tile) * tile
            up, gate = _act(w.detach()).chunk(2, dim=0)
            pad_rows = up.new_zeros(padded - hidden, up.shape[1])
            w_ug = torch.cat([up, pad_rows, gate, pad_rows], dim=0)
            w_down = torch.cat([_act(wd.detach()), wd.new_zeros(wd.shape[0], padded - hidden, dtype=w_ug.dtype)],
                               dim=1).contiguous()
            self._fw = (gemm.interleave_up_gate(w_ug, tile), w_down, tile)
            self._fw_key = key
        return self._fw

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """down(silu(gate) * up): the tcgen05 GEMM with the SwiGLU epilogue, then the down projection."""
        if _wants_grad(self, x):  # reference train/train_dwarf.py:238-240
            up, gate = self.up_gate(x).chunk(2, dim=-1)
            return self.down(self.dropout(F.silu(gate) * up))
        w_il, w_down, tile = self._fused_weights()
        h = gemm.linear_swiglu(_act(x), w_il, tile)
        return gemm.linear(h, w_down)

    def forward_add_rmsnorm(self, x: torch.Tensor, residual: torch.Tensor, norm_weight: torch.Tensor,
                            eps: float = 1e-6) -> tuple[torch.Tensor, torch.Tensor]:
        """(residual + ffn(x), RMSNorm of that * norm_weight) with the residual add and the next
        norm fused into the down projection's epilogue; the residual stream is updated in place."""
        w_il, w_down, tile = self._fused_weights()
        h = gemm.linear_swiglu(_act(x), w_il, tile)
        return gemm.linear_add_rmsnorm(h, w_down, residual, norm_weight, eps=eps, x_out=residual)


class InterferencePacket(nn.Module):
    """Causal EMA packet feeding HISA's global K/V (reference :243-284)."""

    def __init__(self, config: DwarfConfig) -> None:
        super().__init__()
        self.heads = config.num_heads
        self.head_dim = config.embedding_dim // config.num_heads
        raw = [inverse_bounded_ema_factor(1.0 / v) for v in config.ema_timescales]
        self.ema_raw = nn.Parameter(torch.tensor(raw, dtype=torch.float32))
        self.mix_logits = nn.Parameter(torch.zeros(len(raw)))
        self.gate_proj = nn.Linear(config.embedding_dim, config.embedding_dim)
        self.kv_proj = nn.Linear(config.embedding_dim, 2 * config.embedding_dim, bias=False)
        with torch.no_grad():
            self.gate_proj.bias.fill_(-2.0)

    @property
    def ema_factors(self) -> torch.Tensor:
        return bounded_ema_factor(self.ema_raw)

    def _constants(self) -> tuple[torch.Tensor, list[float]]:
        """EMA factors (device) and the bf16 mixture weights (host floats), recomputed only when
        ema_raw or mix_logits change, so a forward needs no device-to-host copy (CUDA-graph safe)."""
        key = (self.ema_raw.data_ptr(), self.ema_raw._version, self.mix_logits.data_ptr(), self.mix_logits._version)
        if getattr(self, "_const_key", None) != key:
            with torch.no_grad():
                factors = self.ema_factors.detach().clone()
                mixture = torch.softmax(self.mix_logits.detach().float(), dim=0).to(torch.bfloat16).float().tolist()
            self._const = (factors, mixture)
            self._const_key = key
        return self._const

    def forward(self, normalized: torch.Tensor, ema_states: list | None = None):
        """(key_delta, value_delta) [B,H,T,hd]. With ``ema_states`` (one fp32 [B,D] state tensor
        per timescale) the scans continue from those states, which are then overwritten in
        place with the states after the last token."""
        if ema_states is None and _wants_grad(self, normalized):
            return self._forward_autograd(normalized)
        x = _act(normalized)
        factors, mixture = self._constants()
        if ema_states is None:
            scans = [causal_ema_scan(x, f.reshape(1)) for f in factors]
        else:
            scans = []
            for f, state in zip(factors, ema_states):
                scan, final = causal_ema_scan(x, f.reshape(1), initial_state=state, return_final_state=True)
                state.copy_(final)
                scans.append(scan)
        gate_pre = gemm.linear(x, _act(self.gate_proj.weight), _act(self.gate_proj.bias))
        packet = glue.packet(scans, mixture, gate_pre)
        kv = gemm.linear(packet, _act(self.kv_proj.weight))
        B, T, D = x.shape
        key_delta = kv[..., :D].reshape(B, T, self.heads, self.head_dim).permute(0, 2, 1, 3)
        value_delta = kv[..., D:].reshape(B, T, self.heads, self.head_dim).permute(0, 2, 1, 3)
        return key_delta, value_delta


def _packet_autograd(self, normalized: torch.Tensor):
    """Differentiable packet (reference train/train_dwarf.py:260-284): the three EMA
    scans on ``causal_ema_scan``'s autograd path, the rest as torch ops."""
    scan_input = normalized.to(torch.bfloat16)
    scans = [causal_ema_scan(scan_input, factor.reshape(1)) for factor in self.ema_factors]
    mixture = torch.softmax(self.mix_logits.float(), dim=0)
    pooled = sum(weight.to(scans[0].dtype) * scan for weight, scan in zip(mixture, scans))
    pooled_float = pooled.float()
    rms = pooled_float.square().mean(-1, keepdim=True).sqrt()
    direction = pooled_float * torch.rsqrt(pooled_float.square().mean(-1, keepdim=True) + 1e-6)
    confidence = torch.tanh(rms / 0.25)
    gate = torch.sigmoid(self.gate_proj(normalized).float())
    packet = (direction * confidence * gate).to(normalized.dtype)
    key_delta, value_delta = self.kv_proj(packet).chunk(2, dim=-1)
    B, T, _ = normalized.shape
    key_delta = key_delta.reshape(B, T, self.heads, self.head_dim).permute(0, 2, 1, 3)
    value_delta = value_delta.reshape(B, T, self.heads, self.head_dim).permute(0, 2, 1, 3)
    return key_delta, value_delta


InterferencePacket._forward_autograd = _packet_autograd


class DSQGBlock(nn.Module):
    def __init__(self, config: DwarfConfig, offsets: tuple[int, ...], *, plane_shift: int,
                 kv_cache: str = "bf16") -> None:
        super().__init__()
        small, large = _small_large_counts(offsets)
        self.norm1 = RMSNorm(config.embedding_dim)
        self.norm2 = RMSNorm(config.embedding_dim)
        self.attn = DSQGAttentionV19(
            config.embedding_dim, config.num_heads, offsets, small, large, seq_len=config.seq_len,
            dropout=config.dropout, grouped_mode="baseline", plane_shift=plane_shift, pos_bias_scale=1.0,
            movt_dynamic_rms_target=0.01, train_phase_probes=False, scale_embed_init_std=0.01,
            npci_strength_tau=0.25, online_softmax=True, support_crop_projections=True,
            support_crop_min_offset=64, kv_cache=kv_cache,
        )
        self.ffn = SwiGLUFFN(config)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if _wants_grad(self, x):  # reference train/train_dwarf.py:320-322
            x = x + self.attn(self.norm1(x))
            return x + self.ffn(self.norm2(x))
        x, n2 = glue.add_rmsnorm(_act(x), self.norm2.weight.detach(), addend=self.attn(self.norm1(x)))
        x, _ = glue.add_rmsnorm(x, self.norm2.weight.detach(), addend=self.ffn(n2))
        return x


class GlobalMixerBlock(nn.Module):
    def __init__(self, config: DwarfConfig) -> None:
        super().__init__()
        self.norm1 = RMSNorm(config.embedding_dim)
        self.norm2 = RMSNorm(config.embedding_dim)
        self.attn = HierarchicalSparseAttentionV16HISACausal(
            D=config.embedding_dim, H=config.num_heads, hd=config.embedding_dim // config.num_heads,
            chunk_size=config.hisa_chunk_size, top_k_chunks=config.top_k_chunks,
            hisa_top_m_tokens=config.hisa_top_m_tokens, local_window=config.hisa_local_window,
            selector_tile_size=config.hisa_selector_tile, representative_mode="mean_max_blend",
            representative_blend_alpha=0.5, route_prior_scale=0.1, route_aux_weight=0.01, route_aux_samples=4,
            route_aux_temperature=1.0, exploration_probability=0.05,
            global_adapter_rank=config.hisa_global_adapter_rank, npci_theta_max=0.25,
            max_seq_len=config.model_length, local_backend="flex", collect_routing_diagnostics=False,
        )
        self.packet = InterferencePacket(config)
        self.ffn = SwiGLUFFN(config)
        self.dropout = nn.Dropout(config.dropout)

    def forward(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        normalized = self.norm1(x)
        attended, auxiliary = self.attn(normalized, kv_inject=self.packet(normalized), return_auxiliary=True)
        if _wants_grad(self, x):  # reference train/train_dwarf.py:356-364
            x = x + self.dropout(attended)
            return x + self.ffn(self.norm2(x)), auxiliary
        x, n2 = glue.add_rmsnorm(_act(x), self.norm2.weight.detach(), addend=attended)
        x, _ = glue.add_rmsnorm(x, self.norm2.weight.detach(), addend=self.ffn(n2))
        return x, auxiliary


@dataclass
class HisaLayerCache:
    """Decode cache of the HISA block: (query, local_key, local_value, global_key,
    global_value) bf16 [B,H,L,64], chunk representatives [B,H,L/64,64], attention
    scratch [B,L,D] and the packet's fp32 EMA states [B,D] (one per timescale)."""

    kv: tuple
    reps: torch.Tensor
    attended: torch.Tensor
    ema: list


@dataclass
class DecodeState:
    """Per-sequence caches of an incremental decode, ``length`` positions filled.

    ``layers[i]`` for a DSQG block: the q6 cache (y, z, k_codes, k_scales, v_codes,
    v_scales) of ``max_len`` positions per (batch, head); for the HISA block a
    ``HisaLayerCache``. ``pos`` is ``length`` on the device (int64 [1]): decode steps
    read it there, so one captured step replays at every position."""

    batch: int
    max_len: int
    length: int
    layers: list
    pos: torch.Tensor


class DecodeGraph:
    """One decode step captured in a CUDA graph and replayed per token.

    Every kernel of the step takes the position from ``state.pos`` on the device and
    the step advances it there, so the same graph serves every position; the host only
    copies the token ids in and replays (one launch instead of ~150). The state must not
    be stepped by other means while a graph is in use, except ``state.length``, which
    ``step`` keeps in sync.
    """

    def __init__(self, model: "DwarfForCausalLM", state: DecodeState) -> None:
        if state.length >= state.max_len:
            raise ValueError("the state is full")
        self.model, self.state = model, state
        device = state.pos.device
        self.ids = torch.zeros(state.batch, dtype=torch.int64, device=device)
        weight = _act(model.embedding.weight.detach()).contiguous()
        self._weight = weight
        torch.cuda.synchronize(device)
        saved = state.pos.clone()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            hidden = model._step_hidden(self.ids, state)
            self.logits = gemm.linear(hidden[:, 0].contiguous(), weight)
        torch.cuda.synchronize(device)
        state.pos.copy_(saved)  # capture records the step; it does not run it

    def step(self, token_ids: torch.Tensor) -> torch.Tensor:
        """Logits [B,V] of ``token_ids`` [B] at position ``state.length`` (a view of the
        graph's output buffer, overwritten by the next step)."""
        state = self.state
        if state.length >= state.max_len:
            raise ValueError(f"the state is full (max_len {state.max_len})")
        self.ids.copy_(token_ids.reshape(-1), non_blocking=True)
        self.graph.replay()
        state.length += 1
        return self.logits


class PrefillGraph:
    """The inference forward of a fixed [batch, seq_len] captured in one CUDA graph.

    ``graph(input_ids)`` copies the ids into the graph's input buffer and replays the
    ~300 kernels of the prefill as one launch, returning the logits [batch, seq_len,
    vocab] (a view of the graph's output buffer, overwritten by the next call). The
    kernels and their arguments are those of ``model(input_ids)`` under
    ``torch.no_grad()`` in eval mode, so the outputs are bit-identical to the eager
    forward's. Weights must not be replaced (re-bound) while a graph is in use;
    in-place updates are seen by the next replay except for the tables the modules
    derive from their parameters (recomputed on the next eager call).
    """

    def __init__(self, model: "DwarfForCausalLM", batch: int, seq_len: int) -> None:
        if model.training:
            raise NotImplementedError("capture_prefill captures the inference forward: call .eval() first")
        device = model.embedding.weight.device
        if device.type != "cuda":
            raise RuntimeError("dwarf_v2_b200 runs on CUDA tensors only (no CPU fallback)")
        self.model = model
        self.ids = torch.full((int(batch), int(seq_len)), 57, dtype=torch.int64, device=device)
        with torch.no_grad():
            model(self.ids)  # eager warm-up: derived tables, workspaces, kernel attributes
        torch.cuda.synchronize(device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.no_grad(), torch.cuda.graph(self.graph):
            self.logits = model(self.ids)
        torch.cuda.synchronize(device)

    def __call__(self, input_ids: torch.Tensor) -> torch.Tensor:
        if tuple(input_ids.shape) != tuple(self.ids.shape):
            raise ValueError(f"this graph was captured for input_ids of shape {tuple(self.ids.shape)}")
        self.ids.copy_(input_ids, non_blocking=True)
        self.graph.replay()
        return self.logits


class DwarfForCausalLM(nn.Module):
    """The 10-block DWARF-v2 language model (reference train/train_dwarf.py:367-470)."""

    def __init__(self, config: DwarfConfig | None = None, *, kv_cache: str = "bf16") -> None:
        super().__init__()
        self.config = config or DwarfConfig()
        config = self.config
        self.kv_cache = kv_cache
        self.offset_groups = build_offset_groups(config)
        self.embedding = nn.Embedding(config.vocab_size, config.embedding_dim)
        self.dropout = nn.Dropout(config.dropout)
        blocks: list[nn.Module] = []
        dsqg_index = 0
        plane_segment = max(2, (config.embedding_dim // config.num_heads) // R_PLANES)
        for group_index in LAYOUT:
            if group_index is None:
                blocks.append(GlobalMixerBlock(config))
                continue
            plane_shift = 2 * (dsqg_index % max(1, plane_segment // 2))
            blocks.append(DSQGBlock(config, self.offset_groups[group_index], plane_shift=plane_shift,
                                    kv_cache=kv_cache))
            dsqg_index += 1
        self.blocks = nn.ModuleList(blocks)
        self.norm = RMSNorm(config.embedding_dim)
        self.lm_head = nn.Linear(config.embedding_dim, config.vocab_size, bias=False)
        self.lm_head.weight = self.embedding.weight
        self.reset_parameters()

    def reset_parameters(self) -> None:
        """Seeded initialisation with the reference's draw order (reference :397-431)."""
        state = torch.random.get_rng_state()
        torch.manual_seed(self.config.init_seed + 20_001)
        try:
            for module in self.modules():
                if isinstance(module, nn.Linear):
                    nn.init.normal_(module.weight, mean=0.0, std=0.02)
                    if module.bias is not None:
                        nn.init.zeros_(module.bias)
                elif isinstance(module, nn.Embedding):
                    nn.init.normal_(module.weight, mean=0.0, std=0.02)
            for module in self.modules():
                if isinstance(module, DSQGAttentionV19):
                    nn.init.normal_(module.phase_base, mean=0.0, std=0.01)
                    nn.init.normal_(module.phase_gain, mean=0.0, std=module.movt_phase_gain_init_std)
                    nn.init.zeros_(module.phase_gate)
                    nn.init.normal_(module.scale_embed, mean=0.0, std=module.scale_embed_init_std)
                    with torch.no_grad():
                        module.scale_embed.sub_(module.scale_embed.mean(0, keepdim=True))
                    module.reset_phase_probes_()
                elif isinstance(module, HierarchicalSparseAttentionV16HISACausal):
                    module.reset_global_adapters_()
                elif isinstance(module, InterferencePacket):
                    with torch.no_grad():
                        module.gate_proj.bias.fill_(-2.0)
        finally:
            torch.random.set_rng_state(state)

    def prepare_runtime(self, device) -> None:
        for module in self.modules():
            if isinstance(module, HierarchicalSparseAttentionV16HISACausal):
                module.prepare_runtime(device, self.config.model_length)

    def _check(self, input_ids: torch.Tensor, *, inference_only: bool = False) -> None:
        if not input_ids.is_cuda:
            raise RuntimeError("dwarf_v2_b200 runs on CUDA tensors only (no CPU fallback)")
        if input_ids.ndim != 2:
            raise ValueError("input_ids must be [B, T]")
        if inference_only and _wants_grad(self):
            raise NotImplementedError("this entry point is inference-only: call .eval() and run under "
                                      "torch.no_grad()")

    def _forward_hidden_autograd(self, input_ids: torch.Tensor):
        """Differentiable forward (training): the reference's forward_hidden
        (train/train_dwarf.py:439-459) -- bf16 activations, as the reference casts them
        on CUDA (its trainer runs under torch.autocast bf16, which these GEMMs expect
        too) -- through the blocks' differentiable paths."""
        x = self.embedding(input_ids).to(torch.bfloat16)
        x = self.dropout(x)
        auxiliary = x.sum() * 0.0
        for block in self.blocks:
            if isinstance(block, GlobalMixerBlock):
                x, block_auxiliary = block(x)
                auxiliary = auxiliary + block_auxiliary
            else:
                x = block(x)
        return self.norm(x).to(torch.bfloat16), auxiliary

    def forward_hidden(self, input_ids: torch.Tensor, *, return_auxiliary: bool = False):
        """Final RMSNorm'd hidden states [B, T, D] (bf16)."""
        self._check(input_ids)
        if _wants_grad(self):
            hidden, auxiliary = self._forward_hidden_autograd(input_ids)
            return (hidden, auxiliary) if return_auxiliary else hidden
        emb = _act(self.embedding.weight.detach()).contiguous()
        blocks = list(self.blocks)
        x, n = glue.embed_rmsnorm(input_ids, emb, blocks[0].norm1.weight.detach())
        auxiliary = x.new_zeros(())
        for i in range(len(blocks)):
            x, n = self._prefill_block(i, x, n)
        return (n, auxiliary) if return_auxiliary else n

    def _prefill_block(self, i: int, x: torch.Tensor, n: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Block ``i`` of the inference prefill: residual stream ``x`` and its norm1 output ``n``
        in; the block output (``x`` is updated in place) and the next norm's output out."""
        blocks = self.blocks
        block = blocks[i]
        next_norm = blocks[i + 1].norm1.weight if i + 1 < len(blocks) else self.norm.weight
        if isinstance(block, GlobalMixerBlock):
            attn = block.attn
            kd, vd = block.packet(n)
            lengths = torch.full((x.shape[0],), x.shape[1], dtype=torch.int32, device=x.device)
            projected, gate, _ = attn.forward_parts(n, (kd, vd), lengths)
            x, n2 = glue.add_rmsnorm(x, block.norm2.weight.detach(), addend=projected, gate=gate)
        else:
            x, n2 = glue.add_rmsnorm(x, block.norm2.weight.detach(), addend=block.attn(n))
        return block.ffn.forward_add_rmsnorm(n2, x, next_norm.detach())

    def prefill_block(self, index: int, x: torch.Tensor) -> torch.Tensor:
        """Output of block ``index`` (reference train/train_dwarf.py:320-322 / :356-364) for the
        residual-stream input ``x`` [B, T, D] bf16, through the fused kernels ``forward_hidden``
        runs (inference only): per-block, teacher-forced parity with the reference's blocks."""
        if not x.is_cuda:
            raise RuntimeError("dwarf_v2_b200 runs on CUDA tensors only (no CPU fallback)")
        if _wants_grad(self):
            raise NotImplementedError("prefill_block is inference-only: call .eval() and run under torch.no_grad()")
        if x.dtype != torch.bfloat16 or x.dim() != 3:
            raise ValueError("prefill_block takes the bf16 residual stream [B, T, D]")
        x = x.contiguous().clone()
        n = glue.rmsnorm(x, self.blocks[index].norm1.weight.detach())
        return self._prefill_block(index, x, n)[0]

    def forward_lse(self, input_ids: torch.Tensor, labels: torch.Tensor | None = None):
        """Per-token (logsumexp, argmax, cross entropy vs ``labels`` or None), each [B, T], from the
        lm_head GEMM's reducing epilogue: the [B, T, vocab] logits are never written."""
        self._check(input_ids, inference_only=True)
        hidden = self.forward_hidden(input_ids)
        B, T, _ = hidden.shape
        lse, argmax, loss = gemm.linear_lse(hidden, _act(self.embedding.weight.detach()),
                                            None if labels is None else labels.reshape(-1))
        shape = (B, T)
        return lse.view(shape), argmax.view(shape), None if loss is None else loss.view(shape)

    # ------------------------------------------------------------------ incremental decoding

    def new_decode_state(self, batch: int, max_len: int | None = None, device=None) -> "DecodeState":
        """Empty per-layer caches for ``batch`` sequences of up to ``max_len`` tokens."""
        if self.kv_cache != "q6":
            raise NotImplementedError("incremental decoding runs on the q6 KV cache (kv_cache='q6')")
        config = self.config
        max_len = int(max_len or config.model_length)
        if max_len < 1 or max_len > 128 * config.hisa_chunk_size:
            raise ValueError(f"max_len must be in [1, {128 * config.hisa_chunk_size}]")
        device = torch.device(device) if device is not None else self.embedding.weight.device
        D = config.embedding_dim
        H, hd = config.num_heads, D // config.num_heads
        layers: list = []
        for block in self.blocks:
            if isinstance(block, GlobalMixerBlock):
                kv = tuple(torch.zeros(batch, H, max_len, hd, dtype=torch.bfloat16, device=device) for _ in range(5))
                chunks = -(-max_len // config.hisa_chunk_size)
                reps = torch.zeros(batch, H, chunks, hd, dtype=torch.bfloat16, device=device)
                attended = torch.zeros(batch, max_len, D, dtype=torch.bfloat16, device=device)
                ema = [torch.zeros(batch, D, dtype=torch.float32, device=device) for _ in config.ema_timescales]
                layers.append(HisaLayerCache(kv, reps, attended, ema))
            else:
                probes = torch.zeros(batch, H, max_len, 4, dtype=torch.float32, device=device)
                codes = torch.zeros(batch, H, max_len, 48, dtype=torch.uint8, device=device)
                scales = torch.zeros(batch, H, max_len, dtype=torch.float16, device=device)
                layers.append((probes, torch.zeros_like(probes), codes, scales, torch.zeros_like(codes),
                               torch.zeros_like(scales)))
        pos = torch.zeros(1, dtype=torch.int64, device=device)
        return DecodeState(batch=batch, max_len=max_len, length=0, layers=layers, pos=pos)

    def forward_cached(self, input_ids: torch.Tensor, state: "DecodeState") -> torch.Tensor:
        """Final RMSNorm'd hidden states [B,T,D] of the T tokens following ``state.length``
        cached positions; appends their caches and advances ``state.length`` by T."""
        self._check(input_ids, inference_only=True)
        B, T = input_ids.shape
        if B != state.batch:
            raise ValueError(f"state holds {state.batch} sequences, input_ids {B}")
        row = state.length
        if row + T > state.max_len:
            raise ValueError(f"{row} cached + {T} new tokens exceed the state's max_len {state.max_len}")
        emb = _act(self.embedding.weight.detach()).contiguous()
        blocks = list(self.blocks)
        x, n = glue.embed_rmsnorm(input_ids, emb, blocks[0].norm1.weight.detach())
        for i, block in enumerate(blocks):
            next_norm = blocks[i + 1].norm1.weight if i + 1 < len(blocks) else self.norm.weight
            layer = state.layers[i]
            if isinstance(block, GlobalMixerBlock):
                kd, vd = block.packet(n, layer.ema)
                projected, gate = block.attn.forward_parts_cached(n, (kd, vd), layer.kv, row)
                # the decode step's running chunk representatives over the whole cache
                lengths = torch.full((B,), row + T, dtype=torch.int32, device=x.device)
                chunk_representatives(layer.kv[3], lengths, blend_alpha=block.attn._blend_alpha, out=layer.reps)
                x, n2 = glue.add_rmsnorm(x, block.norm2.weight.detach(), addend=projected, gate=gate)
            else:
                x, n2 = glue.add_rmsnorm(x, block.norm2.weight.detach(),
                                         addend=block.attn.forward_cached(n, layer, row))
            x, n = block.ffn.forward_add_rmsnorm(n2, x, next_norm.detach())
        state.length = row + T
        state.pos.fill_(state.length)
        return n

    def _step_hidden(self, token_ids: torch.Tensor, state: "DecodeState") -> torch.Tensor:
        """One token per sequence at the device position ``state.pos`` (advanced by one on the
        device); no host value of the position is used, so this is what a CUDA graph captures."""
        B = token_ids.shape[0]
        emb = _act(self.embedding.weight.detach()).contiguous()
        blocks = list(self.blocks)
        x, n = glue.embed_rmsnorm(token_ids.reshape(B, 1), emb, blocks[0].norm1.weight.detach())
        pos = state.pos
        lengths = (pos + 1).to(torch.int32).expand(B).contiguous()
        for i, block in enumerate(blocks):
            next_norm = blocks[i + 1].norm1.weight if i + 1 < len(blocks) else self.norm.weight
            layer = state.layers[i]
            if isinstance(block, GlobalMixerBlock):
                kd, vd = block.packet(n, layer.ema)
                projected, gate = block.attn.forward_step(n, (kd, vd), layer.kv, layer.reps, layer.attended, pos,
                                                          lengths)
                x, n2 = glue.add_rmsnorm(x, block.norm2.weight.detach(), addend=projected, gate=gate)
            else:
                x, n2 = glue.add_rmsnorm(x, block.norm2.weight.detach(), addend=block.attn.forward_step(n, layer, pos))
            x, n = block.ffn.forward_add_rmsnorm(n2, x, next_norm.detach())
        pos.add_(1)
        return n

    def prefill(self, input_ids: torch.Tensor, max_len: int | None = None) -> tuple[torch.Tensor, "DecodeState"]:
        """Prefill ``input_ids`` [B,T] into a new decode state; returns (logits of the last
        token [B,V], state)."""
        state = self.new_decode_state(input_ids.shape[0], max_len, input_ids.device)
        hidden = self.forward_cached(input_ids, state)
        return gemm.linear(hidden[:, -1].contiguous(), _act(self.embedding.weight.detach())), state

    def decode_step(self, state: "DecodeState", token_ids: torch.Tensor) -> torch.Tensor:
        """One incremental step: ``token_ids`` [B] at position ``state.length``; returns its
        logits [B,V] (those of a prefill over the ``state.length + 1`` tokens at its last row,
        up to the decode DSQG kernel's fp32 summation order)."""
        self._check(token_ids.reshape(-1, 1), inference_only=True)
        if token_ids.numel() != state.batch:
            raise ValueError(f"state holds {state.batch} sequences, got {token_ids.numel()} tokens")
        if state.length >= state.max_len:
            raise ValueError(f"the state is full (max_len {state.max_len})")
        hidden = self._step_hidden(token_ids.reshape(-1), state)
        state.length += 1
        return gemm.linear(hidden[:, 0].contiguous(), _act(self.embedding.weight.detach()))

    def capture_prefill(self, batch: int, seq_len: int) -> PrefillGraph:
        """A CUDA graph of the inference prefill of [batch, seq_len] token ids (see PrefillGraph)."""
        return PrefillGraph(self, batch, seq_len)

    def capture_decode(self, state: "DecodeState") -> "DecodeGraph":
        """A CUDA graph of one decode step over ``state``'s buffers (see DecodeGraph)."""
        return DecodeGraph(self, state)

    def check_device_status(self) -> None:
        """Raise ``DeviceTimeoutError`` if a kernel of this model's device hit its bounded-wait
        limit since the last check (the outputs of the launches since then are invalid).
        Synchronises with the device; call it after a forward, not inside a captured graph."""
        _lib.check_device_status(self.embedding.weight.device)

    def forward(self, input_ids: torch.Tensor, *, return_hidden: bool = False, return_auxiliary: bool = False):
        hidden, auxiliary = self.forward_hidden(input_ids, return_auxiliary=True)
        if return_hidden:
            output = hidden
        elif hidden.requires_grad:
            output = self.lm_head(hidden)  # reference train/train_dwarf.py:469
        else:
            output = gemm.linear(hidden, _act(self.embedding.weight.detach()))
        return (output, auxiliary) if return_auxiliary else output
