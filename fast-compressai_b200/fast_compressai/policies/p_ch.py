"""P_ch (channels per coding chunk) selection for the warp_div coder.

The rule is the reference's (policies/p_ch.py:35-88), restated: each
measured candidate has the codec time (encode + decode) and the inference
time (analysis + synthesis transforms) of the same compress / decompress
calls.  A candidate is balanced when its codec / inference ratio is within
``relative_tolerance`` of 1, i.e. the coder keeps pace with the transforms.
The largest balanced P_ch wins (a larger P_ch gives fewer, longer chunks and
a smaller payload); with no balanced candidate, the one whose ratio is
closest to 1 wins, ties going to the larger P_ch.  A plateau diagnostic
marks the first run of ``plateau_patience`` consecutive candidates (in P_ch
order) whose codec times differ by at most ``plateau_delta`` (relative): a
larger P_ch there no longer changes the coder's cost measurably.  The
diagnostic does not affect the choice.  Status and reason strings are the
reference's, so reports and saved selections read the same.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Mapping, Sequence


@dataclass(frozen=True)
class PChSelection:
    selected_p_ch: int
    status: str
    reason: str
    relative_error: float
    plateau: Mapping[str, object]


def legal_p_candidates(channel_count: int, candidates: Sequence[int] | None = None) -> tuple[int, ...]:
    """The distinct integer candidates in [1, channel_count], ascending (all of
    them when ``candidates`` is None).  Non-integers (bool included) are
    dropped; an empty result is an error."""
    if type(channel_count) is not int or channel_count < 1:
        raise ValueError("channel_count must be a positive integer")
    pool = range(1, channel_count + 1) if candidates is None else candidates
    legal = sorted({p for p in pool if type(p) is int and 1 <= p <= channel_count})
    if not legal:
        raise ValueError("no legal P_ch candidates")
    return tuple(legal)


def _positive_time(item: Mapping[str, object], key: str) -> float:
    value = item.get(key)
    if isinstance(value, bool) or not isinstance(value, (int, float)):
        raise ValueError(f"{key} must be a finite positive number")
    value = float(value)
    if not math.isfinite(value) or value <= 0:
        raise ValueError(f"{key} must be a finite positive number")
    return value


def _plateau(points, delta: float, patience: int) -> dict:
    """Pairs of neighbouring candidates with their relative codec-time change,
    and the first run of ``patience`` pairs at or below ``delta``."""
    pairs = [
        {"from_p_ch": a[0], "to_p_ch": b[0], "relative_delta": abs(b[3] - a[3]) / max(a[3], 1e-12)}
        for a, b in zip(points, points[1:])
    ]
    result: dict = {"detected": False, "pairs": pairs}
    run = 0
    for pair in pairs:
        run = run + 1 if pair["relative_delta"] <= delta else 0
        if run >= patience:
            at = pairs.index(pair)  # first pair equal to this one
            result.update(detected=True, start_p_ch=pairs[at - run + 1]["from_p_ch"], end_p_ch=pair["to_p_ch"],
                          interpretation="algorithmic improvement is not distinguishable from measurement variation")
            break
    return result


def choose_p_ch(measurements: Sequence[Mapping[str, object]], *, relative_tolerance: float = 0.10,
                plateau_delta: float = 0.05, plateau_patience: int = 2) -> PChSelection:
    """Choose P_ch from ``measurements`` (mappings with ``p_ch``,
    ``inference_total_ms`` and ``codec_total_ms``); entries whose ``p_ch`` is
    not a positive integer are skipped."""
    if not 0 <= relative_tolerance < 1:
        raise ValueError("relative_tolerance must be in [0, 1)")
    if not 0 <= plateau_delta:
        raise ValueError("plateau_delta must be non-negative")
    if type(plateau_patience) is not int or plateau_patience < 1:
        raise ValueError("plateau_patience must be positive")
    points = []  # (p_ch, codec / inference, |ratio - 1|, codec_ms)
    for item in measurements:
        p = item.get("p_ch")
        if type(p) is not int or p < 1:
            continue
        inference = _positive_time(item, "inference_total_ms")
        codec = _positive_time(item, "codec_total_ms")
        ratio = codec / inference
        points.append((p, ratio, abs(ratio - 1.0), codec))
    if not points:
        raise ValueError("no usable P_ch measurements")
    points.sort()
    plateau = _plateau(points, plateau_delta, plateau_patience)
    balanced = [pt for pt in points if pt[2] <= relative_tolerance]
    if balanced:
        best = max(balanced, key=lambda pt: pt[0])
        return PChSelection(best[0], "auto_selected", "largest_relative_error_pass", best[2], plateau)
    best = min(points, key=lambda pt: (pt[2], -pt[0]))
    return PChSelection(best[0], "fallback_closest_balance", "no_candidate_within_relative_tolerance", best[2],
                        plateau)
