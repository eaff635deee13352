"""Seeded FactorizedPrior inputs shared by the GPU tests and bench.py.

``smooth_images`` is BASELINE config 2's image recipe (seeded Gaussian noise,
5 x 5 box blur, per-image min-max to [0, 1]).  ``spread_latent_prior`` makes a
random-init FactorizedPrior whose latents span its CDF tables: a random-init
analysis transform gives |y| < 0.2, which quantises to all-zero symbols, so
neither the coder nor a transform's rounding error would show at the model
level.  The last analysis convolution is scaled so that y has a chosen
standard deviation, the first synthesis convolution by the inverse (the
synthesis then sees the same signal, quantised on a finer grid), and the
entropy bottleneck's quantiles are set per channel from the latent's median
and range, so that its 16-bit tables cover most of the values and the outer
tail takes the escape (bypass) path.  These are synthetic stand-ins: no
dataset or trained weights are read.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def smooth_images(B: int, H: int, W: int, seed: int, device="cpu") -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, 3, H, W, generator=g)
    x = F.avg_pool2d(F.pad(x, (2, 2, 2, 2), mode="reflect"), 5, stride=1)
    lo = x.amin(dim=(1, 2, 3), keepdim=True)
    hi = x.amax(dim=(1, 2, 3), keepdim=True)
    return ((x - lo) / (hi - lo)).to(device)


@torch.no_grad()
def spread_latent_prior(N: int, M: int, images: torch.Tensor, target_std: float = 6.0, tail: float = 0.9,
                        seed: int = 0):
    """A FactorizedPrior(N, M) on ``images.device`` whose latent of ``images``
    has standard deviation ``target_std``; the CDF tables of channel c cover
    ``median_c + tail * (range_c - median_c)``, the rest escapes."""
    from fast_compressai.balle import FactorizedPrior

    torch.manual_seed(seed)
    model = FactorizedPrior(N, M).to(images.device).eval()
    y = model.g_a(images)
    gain = target_std / float(y.std())
    last, first = model.g_a[6], model.g_s[0]
    last.weight.mul_(gain)
    last.bias.mul_(gain)
    first.weight.div_(gain)
    y = (y * gain).transpose(0, 1).reshape(M, -1)
    med = y.median(dim=1).values
    q = model.entropy_bottleneck.quantiles
    q[:, 0, 0] = med + (y.amin(dim=1) - med) * tail
    q[:, 0, 1] = med
    q[:, 0, 2] = med + (y.amax(dim=1) - med) * tail
    model.update(force=True)
    return model
