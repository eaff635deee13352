"""Generate the golden warp_div fixtures from the reference's own extension.

Runs on a machine with a B200 and oracle/_ref/_warp_div_ref.so (built from
the reference sources by oracle/build_ref.py).  For each case the seeded
inputs are encoded by the reference, and inputs plus outputs are written to
``<out>/<case>.npz``; the reference leaves the header pad bytes
uninitialised, so they are stored as zeros together with a mask.  The
committed fixtures pin the CPU oracle (tests/test_oracle_golden.py).

    python tests/golden/make_golden.py --out tests/golden
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import build_ref  # noqa: E402
from oracle import oracle as O  # noqa: E402
from tests.coder_inputs import channel_indexes, laplacian_symbols, laplacian_tables, small_tables  # noqa: E402

CASES = {
    # name: (B, C, HW, P, escape_rate, explicit random indexes)
    "ref_small_p1": "small:1",
    "ref_small_p2_escape": "small_escape:2",
    "lap_b2_c12_hw16_p5": (2, 12, 16, 5, 0.02, False),
    "lap_b3_c7_hw33_p3": (3, 7, 33, 3, 0.05, False),
    "lap_b1_c4_hw1_p1": (1, 4, 1, 1, 0.3, False),
    "lap_b2_c192_hw48_p4": (2, 192, 48, 4, 0.001, False),
    "lap_b1_c192_hw48_p192": (1, 192, 48, 192, 0.0, False),
    "rand_idx_b2_c9_hw40_p2": (2, 9, 40, 2, 0.0, True),
}


def case_inputs(name):
    spec = CASES[name]
    if isinstance(spec, str):
        kind, p = spec.split(":")
        cdfs, sizes, offs = small_tables()
        base = [0, 1, 2, 3] if kind == "small" else [-100, 100, -101, 102]
        sym = np.array([base * 16], dtype=np.int32)
        idx = np.array([[0, 1, 2, 3] * 16], dtype=np.int32)
        return sym, idx, cdfs, sizes, offs, int(p)
    B, C, HW, P, esc, rand_idx = spec
    cdfs, sizes, offs, scales = laplacian_tables(C, seed=C * 13 + P)
    if rand_idx:
        rng = np.random.default_rng(B + C)
        sym = rng.integers(-45, 45, size=(B, C * HW)).astype(np.int32)
        idx = rng.integers(0, C, size=(B, C * HW)).astype(np.int32)
    else:
        sym = laplacian_symbols(B, C, HW, scales, seed=B * 17 + HW, escape_rate=esc)
        idx = channel_indexes(B, C, HW)
    return sym, idx, cdfs, sizes, offs, P


def main(argv=None) -> int:
    import torch

    ap = argparse.ArgumentParser()
    ap.add_argument("--out", type=Path, required=True)
    args = ap.parse_args(argv)
    args.out.mkdir(parents=True, exist_ok=True)
    ref = build_ref.load()
    dev = torch.device("cuda:0")
    for name in CASES:
        sym, idx, cdfs, sizes, offs, P = case_inputs(name)
        t = [torch.from_numpy(a).to(dev) for a in (sym, idx, cdfs, sizes, offs)]
        packed, mr, hb, cl, p = ref.encode_warp_div(*t, P)
        packed = packed.cpu().numpy().copy()
        hb = int(hb[0])
        mask = O.header_mask(packed.size, hb, mr.numel())
        packed[~mask] = 0
        np.savez_compressed(args.out / f"{name}.npz", symbols=sym, indexes=idx, cdfs=cdfs, cdf_sizes=sizes,
                            offsets=offs, p_ch=P, packed=packed, mask=mask,
                            max_rounds=mr.cpu().numpy().astype(np.uint32), header_bytes=hb,
                            chunk_len=int(cl[0]))
        print(name, packed.size, "bytes")
    return 0


if __name__ == "__main__":
    sys.exit(main())
