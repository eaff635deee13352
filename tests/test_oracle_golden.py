"""Pins the CPU oracle to the reference: the oracle's payloads must equal the
golden fixtures that the reference's own extension produced on a B200
(tests/golden/make_golden.py), byte for byte outside the uninitialised
header pad, and must decode back to the fixture symbols."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"
FIXTURES = sorted(GOLDEN.glob("*.npz"))


def test_golden_fixtures_present():
    assert len(FIXTURES) >= 6, "golden fixtures missing: run tests/golden/make_golden.py on a B200"


@pytest.mark.parametrize("path", FIXTURES, ids=[p.stem for p in FIXTURES])
def test_oracle_matches_reference_fixture(path):
    f = np.load(path)
    packed, mr, hb, cl = O.warp_div_encode(f["symbols"], f["indexes"], f["cdfs"], f["cdf_sizes"], f["offsets"],
                                           int(f["p_ch"]))
    assert hb == int(f["header_bytes"]) and cl == int(f["chunk_len"])
    assert np.array_equal(mr, f["max_rounds"])
    assert packed.size == f["packed"].size
    mask = f["mask"]
    assert np.array_equal(packed[mask], f["packed"][mask])
    dec = O.warp_div_decode(f["packed"], f["max_rounds"], hb, cl, f["indexes"], f["cdfs"], f["cdf_sizes"],
                            f["offsets"])
    assert np.array_equal(dec, f["symbols"])
