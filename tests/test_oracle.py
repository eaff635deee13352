"""CPU tests of the oracle (oracle/warp_div_oracle.c): round trips on the
reference's own known-answer inputs and on seeded random inputs, format
invariants, and the single-stream coder used as the CPU baseline."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from tests.coder_inputs import channel_indexes, laplacian_symbols, laplacian_tables, small_tables


def _roundtrip(symbols, indexes, cdfs, sizes, offsets, P):
    packed, mr, hb, cl = O.warp_div_encode(symbols, indexes, cdfs, sizes, offsets, P)
    dec = O.warp_div_decode(packed, mr, hb, cl, indexes, cdfs, sizes, offsets,
                            batch=symbols.shape[0], symbols_per_batch=symbols.shape[1])
    assert np.array_equal(dec, symbols)
    return packed, mr, hb, cl


@pytest.mark.parametrize("P", [1, 2, 4])
def test_reference_known_answer_round_trip(P):
    # tests/gpu/test_warp_div_cuda.py:18-35 of the reference
    cdfs, sizes, offsets = small_tables()
    symbols = np.array([[0, 1, 2, 3] * 16], dtype=np.int32)
    indexes = np.array([[0, 1, 2, 3] * 16], dtype=np.int32)
    packed, mr, hb, cl = _roundtrip(symbols, indexes, cdfs, sizes, offsets, P)
    assert mr.shape == (1, 4 // P)
    assert hb == 48 and cl == 16 * P


def test_reference_escape_round_trip():
    cdfs, sizes, offsets = small_tables()
    symbols = np.array([[-100, 100, -101, 102] * 16], dtype=np.int32)
    indexes = np.array([[0, 1, 2, 3] * 16], dtype=np.int32)
    _roundtrip(symbols, indexes, cdfs, sizes, offsets, 2)


def test_header_layout():
    cdfs, sizes, offsets, scales = laplacian_tables(12, seed=3)
    sym = laplacian_symbols(3, 12, 16, scales, seed=4)
    packed, mr, hb, cl = _roundtrip(sym, None, cdfs, sizes, offsets, 5)
    h = packed[:32].view(np.uint32)
    K = mr.shape[1]
    assert K == 3 and cl == 5 * 16
    assert h[0] == 12 * 16 and h[1] == cl and h[2] == (K | (3 << 16)) and h[3] == (2 | (32 << 16))
    assert (h[4:8] == 0).all()
    assert np.array_equal(packed[32:32 + 4 * 3 * K].view(np.int32), mr.reshape(-1).astype(np.int32))
    assert hb == (32 + 4 * 3 * K + 15) // 16 * 16
    assert packed.size == hb + 128 * int(mr.sum())
    assert (mr >= 2).all()


@pytest.mark.parametrize(
    "B,C,HW,P,esc",
    [(1, 12, 16, 4, 0.0), (2, 12, 16, 5, 0.01), (2, 7, 33, 3, 0.05), (1, 4, 1, 1, 0.3), (3, 16, 100, 16, 0.0),
     (2, 192, 48, 48, 0.001), (1, 5, 7, 2, 0.5)],
)
def test_random_round_trip(B, C, HW, P, esc):
    cdfs, sizes, offsets, scales = laplacian_tables(C, seed=B * 1000 + C)
    sym = laplacian_symbols(B, C, HW, scales, seed=HW, escape_rate=esc)
    idx = channel_indexes(B, C, HW)
    a = _roundtrip(sym, idx, cdfs, sizes, offsets, P)
    b = _roundtrip(sym, None, cdfs, sizes, offsets, P)
    # implicit channel indexes give the identical payload
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


def test_arbitrary_index_tables():
    rng = np.random.default_rng(5)
    cdfs, sizes, offsets, _ = laplacian_tables(6, seed=7)
    sizes = sizes.copy()
    sizes[2] = 10  # a shorter row: symbols beyond it escape
    cdfs[2, 10:] = 0
    cdfs[2, 9] = 65536
    sym = rng.integers(-40, 40, size=(2, 6 * 20)).astype(np.int32)
    idx = rng.integers(0, 6, size=(2, 6 * 20)).astype(np.int32)
    _roundtrip(sym, idx, cdfs, sizes, offsets, 4)


def test_extreme_values_wrap_like_the_device():
    cdfs, sizes, offsets = small_tables()
    big = np.array([[2**31 - 1, -(2**31), 2**30, -(2**30) - 5] * 8], dtype=np.int32)
    idx = np.array([[0, 1, 2, 3] * 8], dtype=np.int32)
    packed, mr, hb, cl = O.warp_div_encode(big, idx, cdfs, sizes, offsets, 1)
    dec = O.warp_div_decode(packed, mr, hb, cl, idx, cdfs, sizes, offsets)
    # values whose escape code has bit 31 set do not round-trip in the format
    # (the decoder shifts an int32 arithmetically, warp_ans_kernel.cu:322)
    ok = np.abs(big.astype(np.int64) - offsets[idx]) < 2**30
    assert np.array_equal(dec[ok], big[ok])


def test_decode_detects_truncation():
    cdfs, sizes, offsets, scales = laplacian_tables(8, seed=1)
    sym = laplacian_symbols(2, 8, 64, scales, seed=2)
    packed, mr, hb, cl = O.warp_div_encode(sym, None, cdfs, sizes, offsets, 2)
    with pytest.raises(O.OracleError):
        O.warp_div_decode(packed[:-128], mr, hb, cl, None, cdfs, sizes, offsets, batch=2, symbols_per_batch=8 * 64)


@pytest.mark.parametrize("threads", [1, 3])
def test_single_stream_round_trip(threads):
    cdfs, sizes, offsets, scales = laplacian_tables(16, seed=11)
    sym = laplacian_symbols(5, 16, 40, scales, seed=12, escape_rate=0.02)
    words, n = O.rans_encode_batch(sym, None, cdfs, sizes, offsets, threads=threads)
    dec = O.rans_decode_batch(words, n, None, cdfs, sizes, offsets, 5, 16 * 40, threads=threads)
    assert np.array_equal(dec, sym)
    # one stream per image is never larger than the 32-lane format
    packed, *_ = O.warp_div_encode(sym, None, cdfs, sizes, offsets, 16)
    assert int(n.sum()) * 4 <= packed.size


def test_invalid_tables_rejected():
    cdfs, sizes, offsets = small_tables()
    sym = np.zeros((1, 8), dtype=np.int32)
    bad = sizes.copy()
    bad[0] = 6  # larger than L
    with pytest.raises(O.OracleError):
        O.warp_div_encode(sym, None, cdfs, bad, offsets, 1)
