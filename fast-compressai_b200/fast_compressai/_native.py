"""Loader of the package's C-ABI library ``_lib/libfcai_b200.so``.

The library holds every CUDA kernel of the package (sm_100a).  There is no
fallback: if it cannot be loaded, callers get ``NativeLibraryError``.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libfcai_b200.so"

# status codes of include/fcai_warp_div.h
FCAI_OK = 0
FCAI_ERR_INVALID = 1
FCAI_ERR_INDEX_RANGE = 2
FCAI_ERR_TABLE = 3
FCAI_ERR_HEADER = 4
FCAI_ERR_ROUNDS = 5
FCAI_ERR_CORRUPT = 6
FCAI_ERR_WORKSPACE = 7
FCAI_ERR_CUDA = 8

# Size of the static device scratch of fcai_warp_div_encode_noalloc
# (FCAI_WARP_DIV_SCRATCH_BYTES in include/fcai_warp_div.h).
WARP_DIV_SCRATCH_BYTES = 16 * 1024 * 1024


class NativeLibraryError(ImportError):
    """The native library is missing or failed to load."""


class NativeCallError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class WarpDivPlan(ctypes.Structure):
    _fields_ = [
        ("chunks", ctypes.c_int32),
        ("chunk_len", ctypes.c_int32),
        ("header_bytes", ctypes.c_int64),
        ("encode_workspace_bytes", ctypes.c_int64),
        ("decode_workspace_bytes", ctypes.c_int64),
        ("max_packed_bytes", ctypes.c_int64),
    ]


class WarpDivEncodeInfo(ctypes.Structure):
    _fields_ = [
        ("packed_bytes", ctypes.c_int64),
        ("header_bytes", ctypes.c_int64),
        ("required_workspace_bytes", ctypes.c_int64),
        ("chunk_len", ctypes.c_int32),
        ("p_ch", ctypes.c_int32),
        ("index_layout_is_channel", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None

_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64

# name -> (restype, argtypes); every symbol include/*.h declares
SIGNATURES: dict[str, tuple] = {
    "fcai_last_error": (ctypes.c_char_p, []),
    "fcai_version": (ctypes.c_char_p, []),
    "fcai_payload_copy_async": (ctypes.c_int, [_P, _P, _I64, _P]),
    "fcai_quantize_e4m3": (ctypes.c_int, [_P, _P, _P, _P, _I32, _I64, _P]),
    "fcai_warp_div_plan_create": (ctypes.c_int, [_I32, _I32, _I32, _I32, ctypes.POINTER(WarpDivPlan)]),
    "fcai_warp_div_encode": (
        ctypes.c_int,
        [_P, _P, _I32, _I32, _P, _I32, _I32, _P, _P, _I32, _P, _I64, _P, ctypes.POINTER(WarpDivEncodeInfo), _P],
    ),
    "fcai_warp_div_encode_latent": (
        ctypes.c_int,
        [_P, _P, _I32, _I32, _P, _I32, _I32, _P, _P, _I32, _P, _I64, _P, ctypes.POINTER(WarpDivEncodeInfo), _P],
    ),
    "fcai_warp_div_encode_latent_submit": (
        ctypes.c_int,
        [_P, _P, _I32, _I32, _P, _I32, _I32, _P, _P, _I32, _P, _I64, _P, _P],
    ),
    "fcai_warp_div_encode_finish": (
        ctypes.c_int,
        [_I32, _I32, _I32, _I32, _I64, ctypes.POINTER(WarpDivEncodeInfo), _P],
    ),
    "fcai_warp_div_decode_latent": (
        ctypes.c_int,
        [_P, _I64, _P, _I32, _I64, _I32, _I32, _I32, _P, _I32, _I32, _P, _P, _P, _P, _P, _I64, _I32, _P],
    ),
    "fcai_warp_div_encode_pack": (ctypes.c_int, [_P, _I64, _I32, _I32, _I32, _I32, _P, _I64, _P]),
    "fcai_warp_div_encode_noalloc": (
        ctypes.c_int,
        [_P, _P, _I32, _I32, _P, _I32, _I32, _P, _P, _I32, _P, _I64, _P, ctypes.POINTER(WarpDivEncodeInfo), _P],
    ),
    "fcai_layer_out_size": (ctypes.c_int, [_P, _I32, _I32, ctypes.POINTER(_I32), ctypes.POINTER(_I32)]),
    "fcai_layer_forward": (ctypes.c_int, [_P, _I32, _I32, _I32, _P, _P, _P, _P]),
    "fcai_nchw_f32_to_nhwc_bf16": (ctypes.c_int, [_P, _P, _I32, _I32, _I32, _I32, _P]),
    "fcai_warp_div_decode": (
        ctypes.c_int,
        [_P, _I64, _P, _I32, _I64, _I32, _P, _I32, _I32, _P, _I32, _I32, _P, _P, _P, _P, _I64, _I32,
         ctypes.POINTER(_I32), _P],
    ),
}


# Kernels launched through this library since import (each C-ABI call
# launches a known number of kernels; the Python wrappers add them here).
LAUNCHES = {"kernels": 0}


def count_launches(n: int) -> None:
    LAUNCHES["kernels"] += n


# Unchecked decodes of at most this many chunks run without the prep kernel
# (kInlineOffsetChunks in warp_div.cu).
INLINE_OFFSET_CHUNKS = 2048

_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_handle(device: torch.device) -> int:
    """The handle of ``device``'s current CUDA stream.  Uses torch's raw
    query where it exists: ``torch.cuda.current_stream(device)`` builds a
    Stream object and costs microseconds on a path that issues launches."""
    if _raw_stream is not None:
        return _raw_stream(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


class _Nothing:
    __slots__ = ()

    def __enter__(self):
        return None

    def __exit__(self, *exc):
        return False


_NOTHING = _Nothing()


def on_device(device: torch.device):
    """``torch.cuda.device(device)``, or a no-op context when ``device`` is
    already the current one (the common case, and a cheaper one)."""
    if device.index is None or device.index == torch.cuda.current_device():
        return _NOTHING
    return torch.cuda.device(device)


def available() -> bool:
    return LIB_PATH.exists()


def lib() -> ctypes.CDLL:
    """Load (once) and return the native library."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise NativeLibraryError(
                    f"native library {LIB_PATH} is not built; run __graft_entry__.build() or "
                    "fast-compressai_b200/build_native.py"
                )
            try:
                handle = ctypes.CDLL(str(LIB_PATH))
            except OSError as exc:
                raise NativeLibraryError(f"cannot load {LIB_PATH}: {exc}") from exc
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(code: int) -> None:
    """Raise NativeCallError for a non-zero status."""
    if code != FCAI_OK:
        msg = lib().fcai_last_error().decode("utf-8", "replace")
        raise NativeCallError(code, msg or f"native call failed with status {code}")
