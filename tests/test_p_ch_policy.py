"""P_ch selection rule (fast_compressai.choose_p_ch) on hand-made
measurements: the reference's cases (tests/test_p_ch.py of the reference:
largest balanced candidate, fallback to the closest balance, plateau
detection, legal candidates) and the edges of the rule (tolerance bounds,
ties, skipped entries, invalid times and parameters)."""

from __future__ import annotations

import math

import pytest

from fast_compressai import PChSelection, choose_p_ch, default_p_candidates, legal_p_candidates


def _m(p, inference, codec):
    return {"p_ch": p, "inference_total_ms": inference, "codec_total_ms": codec}


def test_legal_candidates_sorted_distinct_and_bounded():
    assert legal_p_candidates(8, [8, 1, 3, 3, 99, 0]) == (1, 3, 8)
    assert legal_p_candidates(3) == (1, 2, 3)
    assert legal_p_candidates(4, [True, 2, 2.0, 4]) == (2, 4)  # bool and float are not P_ch values
    with pytest.raises(ValueError, match="no legal P_ch candidates"):
        legal_p_candidates(4, [0, 5])
    for bad in (0, -1, 2.0, True):
        with pytest.raises(ValueError, match="channel_count must be a positive integer"):
            legal_p_candidates(bad)


def test_default_candidates_follow_the_channel_count():
    assert default_p_candidates(192) == (1, 2, 3, 4, 6, 8, 12, 16, 24, 32, 48, 64, 96, 128, 192)
    assert default_p_candidates(12) == (1, 2, 3, 4, 6, 8, 12)
    assert default_p_candidates(320)[-1] == 256


def test_largest_balanced_candidate_wins():
    r = choose_p_ch([_m(1, 10.0, 30.0), _m(2, 10.0, 10.8), _m(4, 10.0, 9.5)])
    assert isinstance(r, PChSelection)
    assert (r.selected_p_ch, r.status, r.reason) == (4, "auto_selected", "largest_relative_error_pass")
    assert r.relative_error == pytest.approx(0.05)


def test_fallback_to_closest_balance():
    r = choose_p_ch([_m(1, 10.0, 20.0), _m(2, 10.0, 15.0)])
    assert (r.selected_p_ch, r.status, r.reason) == (2, "fallback_closest_balance",
                                                     "no_candidate_within_relative_tolerance")
    assert r.relative_error == pytest.approx(0.5)


def test_fallback_tie_goes_to_the_larger_p():
    # ratios 0.5 and 1.5 are equally far from 1
    r = choose_p_ch([_m(1, 10.0, 5.0), _m(3, 10.0, 15.0), _m(2, 10.0, 40.0)])
    assert r.selected_p_ch == 3 and r.status == "fallback_closest_balance"


def test_tolerance_is_inclusive_and_adjustable():
    ms = [_m(1, 10.0, 11.0), _m(2, 10.0, 12.0)]
    assert choose_p_ch(ms, relative_tolerance=0.2).selected_p_ch == 2
    assert choose_p_ch(ms, relative_tolerance=0.15).selected_p_ch == 1
    assert choose_p_ch(ms, relative_tolerance=0.0).status == "fallback_closest_balance"


def test_plateau_detected_with_its_range():
    ms = [_m(1, 10.0, 30.0), _m(2, 10.0, 20.0), _m(4, 10.0, 19.5), _m(8, 10.0, 19.3)]
    r = choose_p_ch(ms, plateau_patience=2)
    assert r.plateau["detected"]
    assert (r.plateau["start_p_ch"], r.plateau["end_p_ch"]) == (2, 8)
    assert [p["from_p_ch"] for p in r.plateau["pairs"]] == [1, 2, 4]
    assert r.plateau["pairs"][0]["relative_delta"] == pytest.approx(1 / 3)
    assert not choose_p_ch(ms, plateau_patience=3).plateau["detected"]
    assert not choose_p_ch(ms, plateau_delta=0.001).plateau["detected"]


def test_unordered_input_and_skipped_entries():
    ms = [_m(8, 10.0, 9.8), {"p_ch": "4", "inference_total_ms": 1.0, "codec_total_ms": 1.0},
          _m(0, 10.0, 10.0), _m(2, 10.0, 10.1), {"p_ch": True, "inference_total_ms": 1, "codec_total_ms": 1}]
    r = choose_p_ch(ms)
    assert r.selected_p_ch == 8
    assert [p["from_p_ch"] for p in r.plateau["pairs"]] == [2]


@pytest.mark.parametrize("bad", [0.0, -1.0, math.inf, math.nan, "1", True, None])
def test_invalid_times_are_rejected(bad):
    with pytest.raises(ValueError, match="codec_total_ms must be a finite positive number"):
        choose_p_ch([_m(1, 10.0, bad)])
    with pytest.raises(ValueError, match="inference_total_ms must be a finite positive number"):
        choose_p_ch([_m(1, bad, 10.0)])


def test_invalid_parameters_and_empty_input():
    with pytest.raises(ValueError, match="relative_tolerance"):
        choose_p_ch([_m(1, 1.0, 1.0)], relative_tolerance=1.0)
    with pytest.raises(ValueError, match="plateau_delta"):
        choose_p_ch([_m(1, 1.0, 1.0)], plateau_delta=-0.1)
    with pytest.raises(ValueError, match="plateau_patience"):
        choose_p_ch([_m(1, 1.0, 1.0)], plateau_patience=0)
    with pytest.raises(ValueError, match="no usable P_ch measurements"):
        choose_p_ch([{"p_ch": 0}])
