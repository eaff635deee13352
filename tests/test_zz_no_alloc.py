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
import json
import os
import subprocess
import sys
import textwrap
from pathlib import Path

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


# Run in a child process, so that the no-allocation call is the first coder
# call of the process and runs on streams that no earlier call has used.
_FRESH_PROCESS = textwrap.dedent("""
    import ctypes, json, sys
    sys.path[:0] = [sys.argv[1], sys.argv[1] + "/fast-compressai_b200"]
    import numpy as np, torch
    from fast_compressai import _native as N
    from oracle import oracle as O
    from tests.coder_inputs import channel_indexes, laplacian_symbols, laplacian_tables

    dev = torch.device("cuda:0")
    B, C, HW, P = 2, 96, 40, 4
    cdfs, sizes, offs, scales = laplacian_tables(C, seed=51)
    sym = laplacian_symbols(B, C, HW, scales, seed=52, escape_rate=0.01)
    d = [torch.from_numpy(np.ascontiguousarray(a)).to(dev) for a in (sym, cdfs, sizes, offs)]
    plan = N.WarpDivPlan()
    lib = N.lib()
    N.check(lib.fcai_warp_div_plan_create(B, C * HW, C, P, ctypes.byref(plan)))
    outs = [(torch.full((plan.max_packed_bytes,), 0x5A, dtype=torch.uint8, device=dev),
             torch.zeros(B * plan.chunks, dtype=torch.int32, device=dev)) for _ in range(2)]
    torch.cuda.synchronize()

    def call(stream, packed, mr):
        info = N.WarpDivEncodeInfo()
        p = lambda t: ctypes.c_void_p(t.data_ptr())
        rc = lib.fcai_warp_div_encode_noalloc(p(d[0]), None, B, C * HW, p(d[1]), C, cdfs.shape[1], p(d[2]),
                                              p(d[3]), P, p(packed), packed.numel(), p(mr), ctypes.byref(info),
                                              ctypes.c_void_p(stream.cuda_stream))
        stream.synchronize()
        return rc, info

    res = {}
    a0 = torch.cuda.memory_allocated(dev)
    rc, info = call(torch.cuda.Stream(dev), *outs[0])     # first coder call of the process
    res["first"] = [rc, torch.cuda.memory_allocated(dev) - a0]
    free0 = torch.cuda.mem_get_info(dev)[0]
    rc2, info2 = call(torch.cuda.Stream(dev), *outs[1])   # another fresh stream
    res["second"] = [rc2, torch.cuda.memory_allocated(dev) - a0, torch.cuda.mem_get_info(dev)[0] - free0]
    want, want_mr, _, _ = O.warp_div_encode(sym, None, cdfs, sizes, offs, P)
    n = info.packed_bytes
    res["match"] = [bool(np.array_equal(o[0][:n].cpu().numpy(), want)) and
                    bool(np.array_equal(o[1].cpu().numpy().view(np.uint32), want_mr.reshape(-1)))
                    for o in outs] + [n == info2.packed_bytes == want.size]
    print(json.dumps(res))
""")


def test_first_call_in_a_fresh_process_on_fresh_streams():
    # The first call of a process on a stream that has seen no coder call is
    # where the other entry points create their per-stream pinned status slot
    # and event; this one must create nothing there, or on a second fresh
    # stream.  Torch's allocator must not move, and the device's free memory
    # must not change across the second call.
    root = Path(__file__).resolve().parents[1]
    env = dict(os.environ, FCAI_SKIP_BUILD="1")
    proc = subprocess.run([sys.executable, "-c", _FRESH_PROCESS, str(root)], capture_output=True, text=True,
                          timeout=600, env=env)
    assert proc.returncode == 0, proc.stderr[-2000:]
    res = json.loads(proc.stdout.strip().splitlines()[-1])
    assert res["first"] == [0, 0], res
    assert res["second"] == [0, 0, 0], res
    assert all(res["match"]), res
