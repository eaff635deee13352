"""Bit-exact parity with the reference's own warp_div extension.

The reference extension is compiled from the reference sources for sm_100a
by oracle/build_ref.py (output oracle/_ref/_warp_div_ref.so, a test-only
checker).  Payload bytes are compared with the pad bytes between the round
table and header_bytes masked: the reference allocates the payload with
torch::empty and never writes them (warp_ans_kernel_v2.cu:280,
warp_ans_kernel.cu:343-369).  Decoders are cross-checked both ways.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from fast_compressai.coders import _warp_div as ext
from oracle import build_ref
from oracle import oracle as O
from tests.coder_inputs import channel_indexes, laplacian_symbols, laplacian_tables, small_tables

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref():
    return build_ref.load()


def _dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def _check(ref, sym, idx, cdfs, sizes, offs, P, device):
    t = [_dev(a, device) for a in (sym, idx, cdfs, sizes, offs)]
    rp, rmr, rhb, rcl, rP = ref.encode_warp_div(*t, P)
    mine = ext.encode(*t, P)
    hb = int(rhb[0])
    assert mine.header_bytes == hb and mine.chunk_len == int(rcl[0]) and int(rP[0]) == P
    assert torch.equal(mine.max_rounds, rmr)
    a, b = mine.packed.cpu().numpy(), rp.cpu().numpy()
    assert a.size == b.size
    mask = O.header_mask(a.size, hb, mine.max_rounds.numel())
    assert np.array_equal(a[mask], b[mask]), f"first diff at byte {np.argmax((a != b) & mask)}"
    # the reference decoder reads this build's payload and vice versa
    hb_t = torch.tensor([hb], dtype=torch.int64)
    cl_t = torch.tensor([mine.chunk_len], dtype=torch.int32)
    p_t = torch.tensor([P], dtype=torch.int32)
    assert torch.equal(ref.decode_warp_div(mine.packed, mine.max_rounds, hb_t, cl_t, p_t, *t[1:]), t[0])
    assert torch.equal(ext.decode_warp_div(rp, rmr, rhb, rcl, rP, *t[1:]), t[0])
    # and the CPU oracle agrees with both
    op, omr, ohb, _ = O.warp_div_encode(sym, idx, cdfs, sizes, offs, P)
    assert np.array_equal(op[mask], b[mask])


@pytest.mark.parametrize("P", [1, 2, 4])
def test_reference_known_answer_inputs(ref, cuda_device, P):
    cdfs, sizes, offs = small_tables()
    idx = np.array([[0, 1, 2, 3] * 16], dtype=np.int32)
    for sym in ([0, 1, 2, 3] * 16, [-100, 100, -101, 102] * 16):
        _check(ref, np.array([sym], dtype=np.int32), idx, cdfs, sizes, offs, P, cuda_device)


@pytest.mark.parametrize(
    "B,C,HW,P,esc",
    [(1, 12, 16, 4, 0.0), (2, 12, 16, 5, 0.02), (3, 7, 33, 3, 0.05), (1, 4, 1, 1, 0.3), (2, 192, 48, 4, 0.001),
     (2, 192, 48, 192, 0.0), (1, 320, 64, 8, 0.0), (4, 192, 1536, 4, 0.0)],
)
def test_payload_matches_reference(ref, cuda_device, B, C, HW, P, esc):
    cdfs, sizes, offs, scales = laplacian_tables(C, seed=C * 7 + P)
    sym = laplacian_symbols(B, C, HW, scales, seed=B * 31 + HW, escape_rate=esc)
    _check(ref, sym, channel_indexes(B, C, HW), cdfs, sizes, offs, P, cuda_device)


def test_arbitrary_indexes_match_reference(ref, cuda_device):
    rng = np.random.default_rng(4)
    cdfs, sizes, offs, _ = laplacian_tables(9, seed=3)
    sym = rng.integers(-45, 45, size=(2, 9 * 40)).astype(np.int32)
    idx = rng.integers(0, 9, size=(2, 9 * 40)).astype(np.int32)
    _check(ref, sym, idx, cdfs, sizes, offs, 2, cuda_device)
