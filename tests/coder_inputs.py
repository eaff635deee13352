"""Seeded coder inputs shared by the tests, the golden-fixture script and bench.py.

Tables follow BASELINE config 3: per channel a discretised Laplacian with a
scale drawn uniformly from [0.1, 8], symbols clamped to [-32, 32], 16-bit
CDFs with up to 66 entries (65 values + the escape symbol), offsets -32.
Symbols are drawn from the same distributions.  ``escape_rate`` replaces a
fraction of the symbols with out-of-table values to exercise the bypass
path.  These are synthetic stand-ins: no dataset is read.
"""

from __future__ import annotations

import numpy as np

PRECISION = 1 << 16


def laplacian_tables(C: int, seed: int = 0, lo: int = -32, hi: int = 32, scale_range=(0.1, 8.0)):
    """(cdfs int32 [C, L], cdf_sizes int32 [C], offsets int32 [C], scales [C])."""
    rng = np.random.default_rng(seed)
    scales = rng.uniform(scale_range[0], scale_range[1], size=C)
    values = np.arange(lo, hi + 1)
    n = values.size  # in-table values; symbol n (index) is the escape
    L = n + 2
    cdfs = np.zeros((C, L), dtype=np.int32)
    for c in range(C):
        pmf = np.exp(-np.abs(values) / scales[c])
        pmf = pmf / pmf.sum() * (1.0 - 1e-6)
        p = np.concatenate([pmf, [1e-6]])
        freq = np.maximum(1, np.floor(p * PRECISION + 0.5)).astype(np.int64)
        diff = int(freq.sum()) - PRECISION
        order = np.argsort(-freq, kind="stable")
        j = 0
        while diff > 0:
            k = order[j % len(order)]
            take = min(diff, int(freq[k]) - 1)
            freq[k] -= take
            diff -= take
            j += 1
        if diff < 0:
            freq[order[0]] -= diff
        cdfs[c, 1:n + 2] = np.cumsum(freq)
    sizes = np.full(C, L, dtype=np.int32)
    offsets = np.full(C, lo, dtype=np.int32)
    return cdfs, sizes, offsets, scales


def laplacian_symbols(B: int, C: int, HW: int, scales, seed: int = 1, lo: int = -32, hi: int = 32,
                      escape_rate: float = 0.0):
    """int32 [B, C*HW] drawn per channel (channel-major layout)."""
    rng = np.random.default_rng(seed)
    u = rng.uniform(-0.5, 0.5, size=(B, C, HW))
    # inverse CDF of a Laplacian, then round to the integer grid
    x = -np.asarray(scales).reshape(1, C, 1) * np.sign(u) * np.log1p(-2.0 * np.abs(u))
    sym = np.clip(np.rint(x), lo, hi).astype(np.int64)
    if escape_rate > 0:
        mask = rng.random(size=sym.shape) < escape_rate
        wild = rng.integers(-5000, 5000, size=sym.shape)
        wild = np.where(wild >= 0, wild + hi + 1, wild + lo)
        sym = np.where(mask, wild, sym)
    return sym.astype(np.int32).reshape(B, C * HW)


def channel_indexes(B: int, C: int, HW: int):
    return np.broadcast_to(np.repeat(np.arange(C, dtype=np.int32), HW), (B, C * HW)).copy()


def small_tables():
    """The hand-built tables of the reference's own round-trip test
    (tests/gpu/test_warp_div_cuda.py:18-24)."""
    cdfs = np.array([[0, 8192, 16384, 32768, 65536]] * 4, dtype=np.int32)
    sizes = np.array([5] * 4, dtype=np.int32)
    offsets = np.array([-2, -1, 0, 1], dtype=np.int32)
    return cdfs, sizes, offsets
