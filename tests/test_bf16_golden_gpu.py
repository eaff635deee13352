"""The tcgen05 transform layers against the reference's own BF16 operators.

tests/golden/transforms/bf16_layers.npz holds, per layer of a seeded FactorizedPrior(128,
192), the output of the reference's ``BF16Conv2d`` / ``BF16ConvTranspose2d`` /
``BF16GDN`` (backends/pytorch/bf16_operators.py:13-60 of the reference) for the
previous reference layer's output as input.  Each kernel here takes that same
input and must land within 2% of each value plus 0.4% of the tensor's largest
magnitude, with a mean deviation under 0.5% of the mean magnitude (a plain fp32
restatement of these kernels' arithmetic uses at most 0.35 of that bound and
0.27% mean deviation).  The margins
cover the reference's extra roundings: it rounds its bias, the conv output,
the GDN norm, its root and the product to bf16 (each up to 2^-9 relative),
where these kernels keep them in fp32 and round once at the output.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from fast_compressai.transforms import _make_layer, _run
from tests.bf16_golden_model import golden_model, layers

pytestmark = pytest.mark.gpu

FIXTURE = Path(__file__).resolve().parent / "golden" / "transforms" / "bf16_layers.npz"


def _bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).float()


def _nhwc(x):
    return x.permute(0, 2, 3, 1).contiguous().to(torch.bfloat16)


@pytest.mark.parametrize("chain", ["g_a", "g_s"])
def test_layers_match_reference_bf16_operators(cuda_device, chain):
    z = np.load(FIXTURE)
    model = golden_model().to(cuda_device)
    cur = torch.from_numpy(z["x" if chain == "g_a" else "y_hat"]).to(cuda_device)
    with torch.no_grad():
        for i, (conv, gdn) in enumerate(layers(model, chain)):
            first = chain == "g_a" and i == 0
            out_f32 = gdn is None  # the latent (g_a) and the image (g_s) leave as fp32 NCHW
            layer = _make_layer(conv, gdn, first=first, out_f32=out_f32, clamp=False)
            out = _run([layer], cur if first else _nhwc(cur), first_is_nchw=first)
            torch.cuda.synchronize()
            mine = out if out_f32 else out.float().permute(0, 3, 1, 2)
            ref = _bf16(z[f"{chain}.{i}"]).to(cuda_device)
            assert mine.shape == ref.shape, (chain, i)
            err = (mine - ref).abs()
            bound = 0.02 * ref.abs() + 4e-3 * ref.abs().max()
            worst = float((err / bound).max())
            mean_dev = float(err.sum() / ref.abs().sum())
            assert worst <= 1.0 and mean_dev <= 5e-3, (chain, i, worst, mean_dev)
            cur = ref  # the next layer takes the reference's output
