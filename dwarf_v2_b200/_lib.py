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
    return torch.cuda.current_stream(device).cuda_stream


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
        ("device_status", c_ptr),
    ]


def _declare(lib: ctypes.CDLL) -> None:
    lib.dwarf_ema_scan_workspace_bytes.restype = c_i64
    lib.dwarf_ema_scan_workspace_bytes.argtypes = [c_i64, c_i64, c_i64, c_i32]
    lib.dwarf_ema_scan.restype = c_i32
    lib.dwarf_ema_scan.argtypes = [ctypes.POINTER(EmaScanArgs), c_ptr]
