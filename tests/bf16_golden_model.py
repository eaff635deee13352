"""The model and inputs of the BF16 per-layer golden fixture.

Shared by tests/golden/make_bf16_golden.py (which runs the reference's BF16
operators over it) and the tests that check the fixture: a
FactorizedPrior(128, 192) built on the CPU from seed 0, with each GDN's
gamma perturbed off the diagonal from seed 5 so that the GDN GEMM mixes
channels.  The analysis chain takes one 3 x 28 x 36 image, the synthesis
chain one 192 x 1 x 2 latent; ragged sizes exercise the kernels' edge
masking.
"""

from __future__ import annotations

import torch

from fast_compressai.balle import GDN, FactorizedPrior

IMAGE_SHAPE = (1, 3, 28, 36)
LATENT_SHAPE = (1, 192, 1, 2)


def golden_model() -> FactorizedPrior:
    torch.manual_seed(0)
    model = FactorizedPrior(128, 192).eval()
    g = torch.Generator().manual_seed(5)
    with torch.no_grad():
        for m in model.modules():
            if isinstance(m, GDN):
                m.gamma.add_(torch.rand(m.gamma.shape, generator=g) * 0.05)
    return model


def layers(model: FactorizedPrior, chain: str) -> list:
    """[(conv or deconv, GDN or None)] of one chain, as the kernels fuse them."""
    mods = list(getattr(model, chain))
    out = []
    i = 0
    while i < len(mods):
        gdn = mods[i + 1] if i + 1 < len(mods) and isinstance(mods[i + 1], GDN) else None
        out.append((mods[i], gdn))
        i += 2 if gdn is not None else 1
    return out


def weight_checksum(model: FactorizedPrior) -> float:
    """A float64 sum over every transform parameter, to detect a change of the seeded weights."""
    total = 0.0
    for chain in ("g_a", "g_s"):
        for p in getattr(model, chain).parameters():
            total += float(p.detach().double().abs().sum())
    return total
