"""ctypes binding of ``libdwarf_b200.so`` (the engine's C ABI, include/dwarf_b200.h).

Every struct here mirrors one ``dwarf_*_args`` struct field for field. Torch is
used only for device memory and the current CUDA stream; pointers cross the
boundary as plain integers. A missing library, or a call without CUDA tensors,
raises: there is no CPU fallback on the product path.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

ABI_VERSION = 1

DWARF_F32 = 0
DWARF_BF16 = 1
DWARF_F16 = 2

_DTYPE_CODES = {torch.float32: DWARF_F32, torch.bfloat16: DWARF_BF16, torch.float16: DWARF_F16}

c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_f32 = ctypes.c_float
c_ptr = ctypes.c_void_p

_lock = threading.Lock()
_library: ctypes.CDLL | None = None


class DwarfStatusError(RuntimeError):
    """A C entry point returned a negative dwarf_status."""


def library_path() -> Path:
    from . import _build

    return _build.LIBRARY_PATH


def load() -> ctypes.CDLL:
    """Load the shared library (building it first if it is stale or absent)."""
    global _library
    if _library is not None:
        return _library
    with _lock:
        if _library is not None:
            return _library
        from . import _build

        path = _build.LIBRARY_PATH
        try:
            path = _build.build()
        except RuntimeError as exc:
            if not path.is_file():
                raise RuntimeError(
                    f"dwarf_v2_b200: CUDA extension {path.name} is missing and could not be built: {exc}"
                ) from exc
        lib = ctypes.CDLL(str(path))
        lib.dwarf_status_string.restype = ctypes.c_char_p
        lib.dwarf_status_string.argtypes = [c_i32]
        lib.dwarf_abi_version.restype = c_i32
        if lib.dwarf_abi_version() != ABI_VERSION:
            raise RuntimeError("libdwarf_b200.so ABI version mismatch; rebuild the extension")
        _declare(lib)
        _library = lib
        return lib


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {dtype}") from None


def ptr(tensor: torch.Tensor | None) -> int | None:
    return None if tensor is None else tensor.data_ptr()


def stream_handle(device: torch.device) -> int:
    """Raw handle of the current stream of ``device`` (what torch.cuda.current_stream returns)."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    return torch._C._cuda_getCurrentRawStream(index)


def check(status: int, what: str) -> None:
    if status == 0:
        return
    message = load().dwarf_status_string(status).decode()
    text = f"{what}: {message} (status {status})"
    if status in (-3, -4, -5, -9):
        raise ValueError(text)
    if status == -6:
        raise TypeError(text)
    raise DwarfStatusError(text)


def require_cuda(*tensors: torch.Tensor | None) -> None:
    for tensor in tensors:
        if tensor is not None and not tensor.is_cuda:
            raise RuntimeError(
                "dwarf_v2_b200 runs on CUDA tensors only (no CPU fallback); got a "
                f"{tensor.device} tensor"
            )


_status_words: dict[int, torch.Tensor] = {}


def device_status_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 word that kernels with bounded waits write on timeout."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    word = _status_words.get(index)
    if word is None:
        word = torch.zeros(1, dtype=torch.int32, device=f"cuda:{index}")
        _status_words[index] = word
    return word


def read_and_clear_device_status(device: torch.device) -> int:
    word = device_status_word(device)
    value = int(word.item())
    word.zero_()
    return value


class DeviceTimeoutError(RuntimeError):
    """A kernel's bounded wait ran out (DWARF_DEVICE_TIMEOUT): its outputs are not valid."""


def check_device_status(device: torch.device | None = None) -> None:
    """Read and clear the device status word(s); raise DeviceTimeoutError if a kernel
    recorded a timed-out wait since the last check. Synchronises with the device.

    ``device=None`` checks every device that has a status word."""
    if device is None:
        indices = sorted(_status_words)
    else:
        indices = [device.index if device.index is not None else torch.cuda.current_device()]
    bad = []
    for index in indices:
        if index in _status_words and read_and_clear_device_status(torch.device("cuda", index)) != 0:
            bad.append(index)
    if bad:
        raise DeviceTimeoutError(
            f"a dwarf_b200 kernel on cuda:{bad} hit its bounded-wait limit (DWARF_DEVICE_TIMEOUT); "
            "the results of the launches since the last check are not valid")


class EmaScanArgs(ctypes.Structure):
    _fields_ = [
        ("version", c_i32), ("dtype", c_i32),
        ("x", c_ptr), ("y", c_ptr),
        ("batch", c_i64), ("seq_len", c_i64), ("width", c_i64),
        ("sxb", c_i64), ("sxn", c_i64), ("sxd", c_i64),
        ("syb", c_i64), ("syn", c_i64), ("syd", c_i64),
        ("alpha", c_ptr), ("alpha_per_channel", c_i32), ("clamp", c_i32),
        ("floor_", c_f32), ("ceiling", c_f32),
        ("workspace", c_ptr), ("workspace_bytes", c_i64),
        ("device_status", c_ptr), ("init_state", c_ptr), ("final_state", c_ptr),
        ("wait_limit", ctypes.c_uint32), ("test_tag_skew", c_i32),
    ]


def _fields(spec: str):
    """Build a ctypes field list from 'name:type, ...' (i32 i64 f32 ptr)."""
    kinds = {"i32": c_i32, "i64": c_i64, "f32": c_f32, "ptr": c_ptr}
    out = []
    for item in spec.replace("\n", " ").split(","):
        item = item.strip()
        if item:
            name, kind = item.split(":")
            out.append((name.strip(), kinds[kind.strip()]))
    return out


class EmaGradAlphaArgs(ctypes.Structure):
    _fields_ = _fields("""version:i32, dtype:i32, x:ptr, y:ptr, g:ptr, batch:i64, seq_len:i64, width:i64,
        sxb:i64, sxn:i64, sxd:i64, syb:i64, syn:i64, syd:i64, sgb:i64, sgn:i64, sgd:i64,
        alpha:ptr, alpha_per_channel:i32, pad_:i32, da:ptr""")


class Q6PackArgs(ctypes.Structure):
    _fields_ = _fields("""version:i32, dtype:i32, x:ptr, B:i64, H:i64, T:i64, sxb:i64, sxh:i64, sxt:i64,
        codes:ptr, scb:i64, sch:i64, sct:i64, scales:ptr, ssb:i64, ssh:i64, sst:i64""")


class Q6UnpackArgs(ctypes.Structure):
    _fields_ = _fields("""version:i32, out_dtype:i32, codes:ptr, B:i64, H:i64, T:i64, scb:i64, sch:i64, sct:i64,
        scales:ptr, ssb:i64, ssh:i64, sst:i64, x:ptr, sxb:i64, sxh:i64, sxt:i64""")


class DsqgFwdArgs(ctypes.Structure):
    _fields_ = _fields("""version:i32, kv_format:i32, B:i64, H:i64, H_kv:i64, N:i64, head_dim:i32,
        J:i32, j_small:i32, j_large:i32, plane_shift:i32, query_start:i32,
        q:ptr, sqb:i64, sqh:i64, sqn:i64, k:ptr, skb:i64, skh:i64, skn:i64, v:ptr, svb:i64, svh:i64, svn:i64,
        k_codes:ptr, k_scales:ptr, v_codes:ptr, v_scales:ptr, ccb:i64, cch:i64, cct:i64, csb:i64, csh:i64, cst:i64,
        offsets:ptr, pos_bias:ptr, spj:i64, sph:i64, scale_embed:ptr, sej:i64, sed:i64,
        phase_base:ptr, sbj:i64, sbh:i64, phase_gain:ptr, sgj:i64, sgh:i64,
        y_pre:ptr, syb:i64, syh:i64, syn:i64, z_pre:ptr, szb:i64, szh:i64, szn:i64,
        out:ptr, sob:i64, soh:i64, son:i64, lse:ptr, slb:i64, slh:i64, sln:i64,
        head_gain:ptr, head_gain_dtype:i32, gate:ptr, sgb_:i64, sgn_:i64, device_status:ptr, row_begin:i64, pos:ptr""")


class DsqgBwdArgs(ctypes.Structure):
    _fields_ = _fields("""version:i32, J:i32, j_small:i32, j_large:i32, plane_shift:i32, query_start:i32,
        B:i64, H:i64, H_kv:i64, N:i64, q:ptr, k:ptr, v:ptr, out:ptr, dout:ptr, lse:ptr, offsets:ptr,
        pos_bias:ptr, scale_embed:ptr, phase_base:ptr, phase_gain:ptr, y_pre:ptr, z_pre:ptr,
        dq:ptr, dk:ptr, dv:ptr, dy_pre:ptr, dz_pre:ptr, ds:ptr, delta:ptr, d_phase_base:ptr, d_phase_gain:ptr""")


class HisaAttnBwdArgs(ctypes.Structure):
    _fields_ = _fields("""version:i32, k_slots:i32, B:i64, H:i64, T:i64, query:ptr, local_key:ptr, local_value:ptr,
        global_key:ptr, global_value:ptr, top_chunk_idx:ptr, route:ptr, lengths:ptr, out:ptr, dout:ptr,
        dq:ptr, d_local_key:ptr, d_local_value:ptr, d_global_key:ptr, d_global_value:ptr, d_route:ptr,
        lse:ptr, delta:ptr""")


class DsqgPrepArgs(ctypes.Structure):
    _fields_ = _fields("""version:i32, pack_q6:i32, B:i64, H:i64, H_kv:i64, N:i64,
        q:ptr, sqb:i64, sqh:i64, sqn:i64, k:ptr, skb:i64, skh:i64, skn:i64, v:ptr, svb:i64, svh:i64, svn:i64,
        q_probe:ptr, k_probe:ptr, y_pre:ptr, z_pre:ptr, k_codes:ptr, k_scales:ptr, v_codes:ptr, v_scales:ptr""")


class NpciArgs(ctypes.Structure):
    _fields_ = _fields("""version:i32, dtype:i32, B:i64, H:i64, N:i64, x:ptr, sxb:i64, sxh:i64, sxn:i64,
        addend:ptr, sab:i64, sah:i64, san:i64, delta:ptr, sdb:i64, sdh:i64, sdn:i64, theta:ptr, tau:f32,
        out:ptr, sob:i64, soh:i64, son:i64""")


class HisaRepsArgs(ctypes.Structure):
    _fields_ = _fields("""version:i32, head_dim:i32, chunk_size:i32, B:i64, H:i64, T:i64, key:ptr,
        skb:i64, skh:i64, skn:i64, lengths:ptr, blend_alpha:f32, reps:ptr, pos:ptr""")


class HisaSelectArgs(ctypes.Structure):
    _fields_ = _fields("""version:i32, head_dim:i32, chunk_size:i32, selector_tile:i32, top_k:i32,
        B:i64, H:i64, T:i64, query:ptr, sqb:i64, sqh:i64, sqn:i64, reps:ptr, lengths:ptr, temperature:f32,
        top_chunk_idx:ptr, logits:ptr, tile_begin:i64, tile_count:i64, pos:ptr""")


class HisaAttnArgs(ctypes.Structure):
    _fields_ = _fields("""version:i32, head_dim:i32, chunk_size:i32, selector_tile:i32, local_window:i32,
        k_slots:i32, B:i64, H:i64, T:i64,
        query:ptr, sqb:i64, sqh:i64, sqn:i64, local_key:ptr, slkb:i64, slkh:i64, slkn:i64,
        local_value:ptr, slvb:i64, slvh:i64, slvn:i64, global_key:ptr, sgkb:i64, sgkh:i64, sgkn:i64,
        global_value:ptr, sgvb:i64, sgvh:i64, sgvn:i64, top_chunk_idx:ptr, route:ptr,
        lengths:ptr, out:ptr, sob:i64, soh:i64, son:i64, tile_begin:i64, tile_count:i64, pos:ptr,
        lse:ptr, device_status:ptr""")


class HisaRouteArgs(ctypes.Structure):
    _fields_ = _fields("""version:i32, head_dim:i32, selector_tile:i32, k_slots:i32, B:i64, H:i64, T:i64, C:i64,
        query:ptr, sqb:i64, sqh:i64, sqn:i64, reps:ptr, top_chunk_idx:ptr, route_scale:ptr, route:ptr,
        tile_begin:i64, tile_count:i64, pos:ptr""")


class AddRmsNormArgs(ctypes.Structure):
    _fields_ = _fields("""version:i32, w_dtype:i32, rows:i64, width:i64, x:ptr, sx:i64, a:ptr, sa:i64,
        g:ptr, sg:i64, x_out:ptr, sxo:i64, w:ptr, eps:f32, n_out:ptr, sno:i64""")


class EmbedRmsNormArgs(ctypes.Structure):
    _fields_ = _fields("""version:i32, w_dtype:i32, rows:i64, width:i64, vocab:i64, ids:ptr, embedding:ptr,
        w:ptr, eps:f32, x_out:ptr, n_out:ptr""")


class SwigluArgs(ctypes.Structure):
    _fields_ = _fields("version:i32, rows:i64, hidden:i64, in_:ptr, sin:i64, out:ptr, sout:i64")


class GateMulArgs(ctypes.Structure):
    _fields_ = _fields("version:i32, rows:i64, width:i64, a:ptr, sa:i64, g:ptr, sg:i64, out:ptr, so:i64")


class PacketArgs(ctypes.Structure):
    _fields_ = [("version", c_i32), ("n_scans", c_i32), ("rows", c_i64), ("width", c_i64),
                ("scans", c_ptr * 3), ("sscan", c_i64), ("mix", c_f32 * 3), ("gate_pre", c_ptr),
                ("sgp", c_i64), ("out", c_ptr), ("so", c_i64)]


class GemmArgs(ctypes.Structure):
    _fields_ = _fields("""version:i32, epilogue:i32, M:i64, N:i64, K:i64, a:ptr, lda:i64, b:ptr, ldb:i64,
        bias:ptr, bias_dtype:i32, swiglu_tile:i32, out:ptr, ldo:i64, device_status:ptr,
        resid:ptr, ldr:i64, norm_w:ptr, norm_w_dtype:i32, eps:f32, n_out:ptr, ldn:i64,
        T:i64, heads:i32, q_probe:ptr, k_probe:ptr, y_pre:ptr, z_pre:ptr, k_codes:ptr, k_scales:ptr,
        v_codes:ptr, v_scales:ptr, cache_len:i64, lse_part:ptr, arg_part:ptr, targets:ptr, target_logit:ptr, pos:ptr""")


class LseReduceArgs(ctypes.Structure):
    _fields_ = _fields("""version:i32, M:i64, parts:i64, vocab:i64, lse_part:ptr, arg_part:ptr, targets:ptr,
        target_logit:ptr, ignore_index:i64, lse:ptr, argmax:ptr, loss:ptr""")


_ENTRY_POINTS = {
    "dwarf_gemm_bf16": GemmArgs,
    "dwarf_lse_reduce": LseReduceArgs,
    "dwarf_hisa_reps": HisaRepsArgs,
    "dwarf_hisa_select": HisaSelectArgs,
    "dwarf_hisa_attn": HisaAttnArgs,
    "dwarf_hisa_attn_bwd": HisaAttnBwdArgs,
    "dwarf_hisa_route": HisaRouteArgs,
    "dwarf_add_rmsnorm": AddRmsNormArgs,
    "dwarf_embed_rmsnorm": EmbedRmsNormArgs,
    "dwarf_swiglu": SwigluArgs,
    "dwarf_gate_mul": GateMulArgs,
    "dwarf_packet": PacketArgs,
    "dwarf_npci_rotate": NpciArgs,
    "dwarf_ema_scan": EmaScanArgs,
    "dwarf_ema_scan_noalloc": EmaScanArgs,
    "dwarf_ema_scan_grad_alpha": EmaGradAlphaArgs,
    "dwarf_q6_pack": Q6PackArgs,
    "dwarf_q6_unpack": Q6UnpackArgs,
    "dwarf_dsqg_fwd": DsqgFwdArgs,
    "dwarf_dsqg_bwd": DsqgBwdArgs,
    "dwarf_dsqg_prep": DsqgPrepArgs,
}


class LaunchLog:
    """Counts C-ABI launches and, for the entry points in `timed`, brackets each
    with CUDA events on the launching (current) stream."""

    def __init__(self, timed: tuple[str, ...] = ()):
        self.count = 0
        self.timed = set(timed)
        self.events: dict[str, list[tuple[torch.cuda.Event, torch.cuda.Event]]] = {n: [] for n in timed}

    def mean_ms(self, name: str) -> float | None:
        pairs = self.events.get(name) or []
        if not pairs:
            return None
        return sum(a.elapsed_time(b) for a, b in pairs) / len(pairs)


_launch_log: LaunchLog | None = None


def set_launch_log(log: LaunchLog | None) -> None:
    global _launch_log
    _launch_log = log


def call(name: str, args: ctypes.Structure, device: torch.device) -> None:
    """Invoke a C entry point on the current stream of `device`; raise on error.

    Entry points with a ``device_status`` field get the device's status word
    when the caller left it null, so every kernel with bounded waits reports a
    timeout where ``check_device_status`` can see it."""
    lib = load()
    if hasattr(args, "device_status") and not args.device_status:
        args.device_status = device_status_word(device).data_ptr()
    log = _launch_log
    if log is None:
        status = getattr(lib, name)(ctypes.byref(args), stream_handle(device))
    else:
        log.count += 1
        if name in log.timed:
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            status = getattr(lib, name)(ctypes.byref(args), stream_handle(device))
            end.record()
            log.events[name].append((start, end))
        else:
            status = getattr(lib, name)(ctypes.byref(args), stream_handle(device))
    check(status, name)


def _declare(lib: ctypes.CDLL) -> None:
    for name, struct in _ENTRY_POINTS.items():
        fn = getattr(lib, name)
        fn.restype = c_i32
        fn.argtypes = [ctypes.POINTER(struct), c_ptr]
    lib.dwarf_ema_scan_workspace_bytes.restype = c_i64
    lib.dwarf_ema_scan_workspace_bytes.argtypes = [c_i64, c_i64, c_i64, c_i32]
