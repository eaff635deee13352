"""ctypes front end of the CPU oracle (oracle/warp_div_oracle.c).

TEST INFRASTRUCTURE ONLY: the checker for the CUDA coder.  It may be used by
tests/, by ``__graft_entry__.smoke()`` and by the CPU-baseline leg of
``bench.py``; the product package never imports it.

Parity pin: ``tests/test_oracle_golden.py`` checks these functions against
payload fixtures produced by the reference's own CUDA extension
(``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_SRC = _HERE / "warp_div_oracle.c"
_LIB = _HERE / "_build" / "liboracle.so"
_lib = None

ORC_EINVAL, ORC_ECAPACITY, ORC_ECORRUPT, ORC_ENOMEM = 1, 2, 3, 4


class OracleError(RuntimeError):
    pass


def build(force: bool = False) -> Path:
    """Compile the oracle with gcc into oracle/_build/liboracle.so."""
    if force or not _LIB.exists() or _LIB.stat().st_mtime < _SRC.stat().st_mtime:
        _LIB.parent.mkdir(parents=True, exist_ok=True)
        tmp = _LIB.with_suffix(f".{os.getpid()}.tmp")
        subprocess.run(
            ["gcc", "-O2", "-fPIC", "-shared", "-std=c11", "-Wall", "-o", str(tmp), str(_SRC), "-lpthread"],
            check=True,
        )
        os.replace(tmp, _LIB)
    return _LIB


def _load():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(str(build()))
        P = ctypes.c_void_p
        i32, i64 = ctypes.c_int32, ctypes.c_int64
        lib.oracle_warp_div_encode.restype = i64
        lib.oracle_warp_div_encode.argtypes = [P, P, i32, i32, P, i32, i32, P, P, i32, P, i64, P]
        lib.oracle_warp_div_decode.restype = ctypes.c_int
        lib.oracle_warp_div_decode.argtypes = [P, i64, P, i64, i32, P, i32, i32, P, i32, i32, P, P, i32, P]
        lib.oracle_warp_div_dims.restype = None
        lib.oracle_warp_div_dims.argtypes = [i32, i32, i32, i32, P, P, P]
        lib.oracle_rans_batch.restype = ctypes.c_int
        lib.oracle_rans_batch.argtypes = [P, P, i32, i32, P, i32, i32, P, P, P, i64, P, P, ctypes.c_int]
        _lib = lib
    return _lib


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def dims(B: int, N: int, C: int, P: int) -> tuple[int, int, int]:
    """(K, chunk_len, header_bytes) of a warp_div payload."""
    k, cl, hb = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int64()
    _load().oracle_warp_div_dims(B, N, C, P, ctypes.byref(k), ctypes.byref(cl), ctypes.byref(hb))
    return k.value, cl.value, hb.value


def warp_div_encode(symbols, indexes, cdfs, cdf_sizes, offsets, p_ch: int):
    """Return (packed uint8, max_rounds uint32 [B,K], header_bytes, chunk_len)."""
    symbols = _i32(symbols)
    idx = None if indexes is None else _i32(indexes)
    cdfs, cdf_sizes, offsets = _i32(cdfs), _i32(cdf_sizes), _i32(offsets)
    B, N = symbols.shape
    C, L = cdfs.shape
    K, chunk_len, header_bytes = dims(B, N, C, p_ch)
    max_rounds = np.zeros((B, K), dtype=np.uint32)
    lib = _load()
    size = lib.oracle_warp_div_encode(_ptr(symbols), _ptr(idx), B, N, _ptr(cdfs), C, L, _ptr(cdf_sizes),
                                      _ptr(offsets), p_ch, None, 0, _ptr(max_rounds))
    if size < 0:
        raise OracleError(f"oracle encode failed ({size})")
    packed = np.zeros(size, dtype=np.uint8)
    size2 = lib.oracle_warp_div_encode(_ptr(symbols), _ptr(idx), B, N, _ptr(cdfs), C, L, _ptr(cdf_sizes),
                                       _ptr(offsets), p_ch, _ptr(packed), size, _ptr(max_rounds))
    if size2 != size:
        raise OracleError(f"oracle encode failed ({size2})")
    return packed, max_rounds, header_bytes, chunk_len


def warp_div_decode(packed, max_rounds, header_bytes: int, chunk_len: int, indexes, cdfs, cdf_sizes, offsets,
                    batch: int | None = None, symbols_per_batch: int | None = None):
    packed = np.ascontiguousarray(np.asarray(packed, dtype=np.uint8))
    max_rounds = np.ascontiguousarray(np.asarray(max_rounds, dtype=np.uint32))
    cdfs, cdf_sizes, offsets = _i32(cdfs), _i32(cdf_sizes), _i32(offsets)
    idx = None if indexes is None else _i32(indexes)
    if idx is not None:
        B, N = idx.shape
    else:
        B, N = batch, symbols_per_batch
    C, L = cdfs.shape
    K = max_rounds.shape[1]
    out = np.zeros((B, N), dtype=np.int32)
    rc = _load().oracle_warp_div_decode(_ptr(packed), packed.size, _ptr(max_rounds), header_bytes, chunk_len,
                                        _ptr(idx), B, N, _ptr(cdfs), C, L, _ptr(cdf_sizes), _ptr(offsets), K,
                                        _ptr(out))
    if rc:
        raise OracleError(f"oracle decode failed ({rc})")
    return out


def rans_encode_batch(symbols, indexes, cdfs, cdf_sizes, offsets, threads: int = 1):
    """Single-stream rANS per image.  Returns (words [B, cap], n_words [B])."""
    symbols = _i32(symbols)
    idx = None if indexes is None else _i32(indexes)
    cdfs, cdf_sizes, offsets = _i32(cdfs), _i32(cdf_sizes), _i32(offsets)
    B, N = symbols.shape
    C, L = cdfs.shape
    cap = 10 * N + 2
    words = np.empty((B, cap), dtype=np.uint32)
    n_words = np.zeros(B, dtype=np.int64)
    rc = _load().oracle_rans_batch(_ptr(symbols), _ptr(idx), B, N, _ptr(cdfs), C, L, _ptr(cdf_sizes),
                                   _ptr(offsets), _ptr(words), cap, _ptr(n_words), None, threads)
    if rc:
        raise OracleError(f"oracle rans encode failed ({rc})")
    return words, n_words


def rans_decode_batch(words, n_words, indexes, cdfs, cdf_sizes, offsets, B: int, N: int, threads: int = 1):
    words = np.ascontiguousarray(words, dtype=np.uint32)
    n_words = np.ascontiguousarray(n_words, dtype=np.int64)
    idx = None if indexes is None else _i32(indexes)
    cdfs, cdf_sizes, offsets = _i32(cdfs), _i32(cdf_sizes), _i32(offsets)
    C, L = cdfs.shape
    out = np.empty((B, N), dtype=np.int32)
    rc = _load().oracle_rans_batch(None, _ptr(idx), B, N, _ptr(cdfs), C, L, _ptr(cdf_sizes), _ptr(offsets),
                                   _ptr(words), words.shape[1], _ptr(n_words), _ptr(out), threads)
    if rc:
        raise OracleError(f"oracle rans decode failed ({rc})")
    return out


def header_mask(packed_size: int, header_bytes: int, n_chunks: int) -> np.ndarray:
    """Boolean mask of the bytes the reference defines (pad bytes excluded)."""
    mask = np.ones(packed_size, dtype=bool)
    mask[32 + 4 * n_chunks:header_bytes] = False
    return mask
