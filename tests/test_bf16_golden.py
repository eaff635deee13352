"""CPU checks of the BF16 per-layer golden fixture (tests/golden/transforms/bf16_layers.npz,
made by tests/golden/make_bf16_golden.py from the reference's BF16 operators):
the seeded model still has the weights the fixture was made with, and every
stored layer output has the shape the layer produces."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

from tests.bf16_golden_model import IMAGE_SHAPE, LATENT_SHAPE, golden_model, layers, weight_checksum

FIXTURE = Path(__file__).resolve().parent / "golden" / "transforms" / "bf16_layers.npz"


def test_fixture_matches_the_seeded_model():
    z = np.load(FIXTURE)
    model = golden_model()
    assert abs(weight_checksum(model) - float(z["weight_checksum"])) <= 1e-9 * float(z["weight_checksum"])
    assert z["x"].shape == IMAGE_SHAPE and z["y_hat"].shape == LATENT_SHAPE
    with torch.no_grad():
        for chain, cur in (("g_a", torch.from_numpy(z["x"])), ("g_s", torch.from_numpy(z["y_hat"]))):
            for i, (conv, gdn) in enumerate(layers(model, chain)):
                cur = conv(cur)
                if gdn is not None:
                    cur = gdn(cur)
                assert z[f"{chain}.{i}"].shape == tuple(cur.shape), (chain, i)
                assert z[f"{chain}.{i}"].dtype == np.uint16  # exact bf16 bit patterns
