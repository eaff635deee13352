"""CPU checks of the C-ABI library: it loads, exports every symbol the public
headers declare, and its host-side validation matches the reference's
preconditions (no GPU call is made here)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from fast_compressai import _native
from oracle import oracle as O

INCLUDE = Path(__file__).resolve().parents[1] / "include"


def _declared_symbols() -> set[str]:
    names = set()
    for header in INCLUDE.glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names.update(re.findall(r"\b(fcai_[a-z0-9_]+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    lib = _native.lib()
    declared = _declared_symbols()
    assert {"fcai_warp_div_encode", "fcai_warp_div_decode", "fcai_warp_div_encode_pack"} <= declared
    for name in declared:
        assert hasattr(lib, name), name
    assert set(_native.SIGNATURES) >= declared
    assert lib.fcai_version().decode().startswith("fcai-b200")


@pytest.mark.parametrize("B,N,C,P", [(1, 64, 4, 1), (24, 192 * 1536, 192, 4), (64, 192 * 1536, 192, 192),
                                     (2, 12 * 16, 12, 5), (3, 7 * 33, 7, 3)])
def test_plan_matches_oracle_sizes(B, N, C, P):
    plan = _native.WarpDivPlan()
    _native.check(_native.lib().fcai_warp_div_plan_create(B, N, C, P, ctypes.byref(plan)))
    K, chunk_len, header = O.dims(B, N, C, P)
    assert (plan.chunks, plan.chunk_len, plan.header_bytes) == (K, chunk_len, header)
    lane = (chunk_len + 31) // 32
    assert plan.max_packed_bytes == header + B * K * 128 * (10 * lane + 2)
    assert plan.encode_workspace_bytes > plan.max_packed_bytes - header


@pytest.mark.parametrize(
    "B,N,C,P,message",
    [
        (0, 64, 4, 1, "empty/invalid coder input dimensions"),
        (1, 65, 4, 1, "divisible by CDF count"),
        (1, 64, 4, 5, "P_ch must be in [1, C]"),
        (1, 64, 4, 0, "P_ch must be in [1, C]"),
        (65536, 64, 4, 1, "B/C exceed WarpANS header field capacity"),
        (1, 40000 * 1000, 40000, 1, "coder dimensions exceed kernel index range"),
    ],
)
def test_plan_rejects_like_the_reference(B, N, C, P, message):
    plan = _native.WarpDivPlan()
    N = min(N, 2**31 - 1)
    code = _native.lib().fcai_warp_div_plan_create(B, N, C, P, ctypes.byref(plan))
    assert code == _native.FCAI_ERR_INVALID
    assert message in _native.lib().fcai_last_error().decode()


def test_encode_validates_before_touching_the_device():
    info = _native.WarpDivEncodeInfo()
    lib = _native.lib()
    code = lib.fcai_warp_div_encode(None, None, 1, 65, None, 4, 5, None, None, 1, None, 0, None,
                                    ctypes.byref(info), None)
    assert code == _native.FCAI_ERR_INVALID
    with pytest.raises(_native.NativeCallError, match="divisible"):
        _native.check(code)
    code = lib.fcai_warp_div_decode(None, 100, None, 1, 16, 16, None, 1, 64, None, 4, 5, None, None, None, None, 0, 1,
                                    None, None)
    assert code == _native.FCAI_ERR_INVALID
    assert "invalid payload metadata" in lib.fcai_last_error().decode()
