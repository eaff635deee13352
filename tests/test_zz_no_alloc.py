"""fcai_warp_div_encode_noalloc against fcai_warp_div_encode + _pack.

The no-allocation entry point encodes through a static device scratch array
that every call shares, so it is checked on consecutive calls of different
shapes and table layouts: each call's payload, round table and info must
equal what the workspace entry points produce for the same inputs (and the
CPU oracle's payload).  Both paths are called through the C ABI with device
pointers.  The file sorts last so that, in a full run, the scratch array has
already seen a process that ran every other test.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from fast_compressai import _native as N
from oracle import oracle as O
from tests.coder_inputs import channel_indexes, laplacian_symbols, laplacian_tables

pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _case(B, C, HW, P, seed, esc, layout, device):
    cdfs, sizes, offs, scales = laplacian_tables(C, seed=seed)
    sym = laplacian_symbols(B, C, HW, scales, seed=seed + 1, escape_rate=esc)
    if layout in ("channel", "none"):  # "none": indexes = NULL, the channel layout implied
        idx = channel_indexes(B, C, HW)
    else:
        idx = np.random.default_rng(seed).integers(0, C, size=(B, C * HW)).astype(np.int32)
    host = dict(sym=sym, idx=idx, cdfs=cdfs, sizes=sizes, offs=offs)
    dev = {k: torch.from_numpy(np.ascontiguousarray(v)).to(device) for k, v in host.items()}
    return dict(B=B, N=C * HW, C=C, L=cdfs.shape[1], P=P, explicit=layout != "none", host=host, dev=dev)


def _plan(c):
    plan = N.WarpDivPlan()
    N.check(N.lib().fcai_warp_div_plan_create(c["B"], c["N"], c["C"], c["P"], ctypes.byref(plan)))
    return plan


def _args(c):
    d = c["dev"]
    return (_ptr(d["sym"]), _ptr(d["idx"]) if c["explicit"] else None, c["B"], c["N"], _ptr(d["cdfs"]), c["C"],
            c["L"], _ptr(d["sizes"]), _ptr(d["offs"]), c["P"])


def _encode_with_workspace(c, device):
    lib = N.lib()
    plan = _plan(c)
    ws = torch.zeros(plan.encode_workspace_bytes, dtype=torch.uint8, device=device)
    mr = torch.empty(c["B"] * plan.chunks, dtype=torch.int32, device=device)
    info = N.WarpDivEncodeInfo()
    N.check(lib.fcai_warp_div_encode(*_args(c), _ptr(ws), ws.numel(), _ptr(mr), ctypes.byref(info), _stream()))
    packed = torch.empty(info.packed_bytes, dtype=torch.uint8, device=device)
    N.check(lib.fcai_warp_div_encode_pack(_ptr(ws), ws.numel(), c["B"], c["N"], c["C"], c["P"], _ptr(packed),
                                          packed.numel(), _stream()))
    torch.cuda.synchronize()
    return packed.cpu().numpy(), mr.cpu().numpy(), info


def _encode_noalloc(c, device, capacity=None, fill=0xA5):
    plan = _plan(c)
    # Stale bytes in both outputs: only what the call writes may survive.
    packed = torch.full((plan.max_packed_bytes,), fill, dtype=torch.uint8, device=device)
    mr = torch.full((c["B"] * plan.chunks,), -7, dtype=torch.int32, device=device)
    info = N.WarpDivEncodeInfo()
    cap = packed.numel() if capacity is None else capacity
    rc = N.lib().fcai_warp_div_encode_noalloc(*_args(c), _ptr(packed), cap, _ptr(mr), ctypes.byref(info),
                                              _stream())
    torch.cuda.synchronize()
    return rc, packed.cpu().numpy(), mr.cpu().numpy(), info


def _info_tuple(info):
    return (info.packed_bytes, info.header_bytes, info.chunk_len, info.p_ch, info.index_layout_is_channel)


def _check_same(c, device):
    want_packed, want_mr, want_info = _encode_with_workspace(c, device)
    rc, packed, mr, info = _encode_noalloc(c, device)
    N.check(rc)
    assert _info_tuple(info) == _info_tuple(want_info)
    assert np.array_equal(mr, want_mr)
    got = packed[: info.packed_bytes]
    assert np.array_equal(got, want_packed), f"first diff at byte {np.argmax(got != want_packed)}"
    h = c["host"]
    ref_packed, ref_mr, _, _ = O.warp_div_encode(h["sym"], h["idx"], h["cdfs"], h["sizes"], h["offs"], c["P"])
    assert np.array_equal(got, ref_packed) and np.array_equal(mr.view(np.uint32), ref_mr.reshape(-1))


def test_consecutive_calls_match_workspace_entry_points(cuda_device):
    # A large call, then a small one whose chunks fall inside the first
    # call's leftovers, then a large one again with another table layout.
    cases = [
        _case(3, 192, 48, 4, seed=11, esc=0.01, layout="channel", device=cuda_device),
        _case(2, 12, 16, 5, seed=12, esc=0.05, layout="random", device=cuda_device),
        _case(2, 192, 64, 3, seed=13, esc=0.002, layout="none", device=cuda_device),
    ]
    for c in cases:
        _check_same(c, cuda_device)


def test_repeated_identical_calls(cuda_device):
    c = _case(2, 64, 40, 8, seed=21, esc=0.02, layout="channel", device=cuda_device)
    first = _encode_noalloc(c, cuda_device, fill=0x00)
    second = _encode_noalloc(c, cuda_device, fill=0xFF)
    N.check(first[0])
    N.check(second[0])
    n = first[3].packed_bytes
    assert n == second[3].packed_bytes
    assert np.array_equal(first[1][:n], second[1][:n]) and np.array_equal(first[2], second[2])
    _check_same(c, cuda_device)


def test_limit_is_the_worst_case_workspace(cuda_device):
    # One image of 192 channels at P_ch=4: 2176 positions per channel is the
    # largest size whose worst-case workspace fits the scratch, 2184 the next
    # size that changes it.
    fits = _case(1, 192, 2176, 4, seed=31, esc=0.001, layout="channel", device=cuda_device)
    over = _case(1, 192, 2184, 4, seed=32, esc=0.001, layout="channel", device=cuda_device)
    assert _plan(fits).encode_workspace_bytes <= N.WARP_DIV_SCRATCH_BYTES < _plan(over).encode_workspace_bytes
    rc, _, mr, info = _encode_noalloc(over, cuda_device)
    assert rc == N.FCAI_ERR_WORKSPACE
    assert "static scratch" in N.lib().fcai_last_error().decode()
    assert info.required_workspace_bytes == _plan(over).encode_workspace_bytes
    assert (mr == -7).all()  # rejected before any device work
    _check_same(fits, cuda_device)


def test_rejects_a_short_payload_buffer_then_recovers(cuda_device):
    c = _case(2, 32, 50, 4, seed=41, esc=0.01, layout="channel", device=cuda_device)
    plan = _plan(c)
    rc, _, _, _ = _encode_noalloc(c, cuda_device, capacity=plan.header_bytes)
    assert rc == N.FCAI_ERR_INVALID
    assert "cannot hold" in N.lib().fcai_last_error().decode()
    _check_same(c, cuda_device)
