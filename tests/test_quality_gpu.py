"""Quality gates of the B200 transforms against the FP32 path, on latents
that span the CDF tables.

The gates are the north star's: a PSNR drop of at most 0.1 dB against the
FP32 transforms, and a payload (bpp) within 1% of the FP32 path's, at the
same P_ch.  The model is ``tests.model_inputs.spread_latent_prior``: a
random-init FactorizedPrior(128, 192) whose latent has a symbol spread of a
few units (with escapes), because a plain random-init one quantises to
all-zero symbols and would pass any gate.  The FP32 path is accelerate's
``transforms="fp32"`` (the model's torch modules) with cuDNN's TF32 off.
Each variant also reports its symbol mismatch rate against the FP32 latent,
the largest latent error relative to the latent's range, and the PSNR of its
reconstruction against the FP32 one.
"""

from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch
import torch.nn.functional as F

from fast_compressai import accelerate
from fast_compressai.configs import model_fingerprint
from tests.model_inputs import smooth_images, spread_latent_prior

pytestmark = pytest.mark.gpu

FIXTURE = Path(__file__).resolve().parent / "golden" / "precision_map_factorized.json"


def _psnr(a, b):
    return float(10 * torch.log10(1.0 / F.mse_loss(a.float(), b.float())))


@pytest.fixture(scope="module")
def fp32_run(cuda_device):
    tf32 = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        x = smooth_images(4, 256, 384, seed=21, device=cuda_device)
        model = spread_latent_prior(128, 192, x, target_std=12.0)
        ref = accelerate(model, P=4, device="cuda:0", transforms="fp32")
        with torch.inference_mode():
            out = ref.compress(x)
            x_ref = ref.decompress(out["strings"], out["shape"])["x_hat"]
            eb = model.entropy_bottleneck
            med = eb._get_medians().detach().reshape(1, -1, 1, 1)
            y_ref = model.g_a(x)
        torch.cuda.synchronize()
    finally:
        torch.backends.cudnn.allow_tf32 = tf32
    return dict(x=x, model=model, bytes=out["strings"][0].packed.numel(), x_ref=x_ref, y_ref=y_ref, med=med)


def _variant(fp32_run, variant, tmp_path):
    model = fp32_run["model"]
    if variant == "precision_map":
        data = json.loads(FIXTURE.read_text())
        data["model_fingerprint"] = model_fingerprint(model)
        data["p_ch"] = 4
        path = tmp_path / "map.json"
        path.write_text(json.dumps(data))
        return accelerate(model, P=4, device="cuda:0", precision_config_path=str(path))
    return accelerate(model, P=4, device="cuda:0", transforms=variant)


@pytest.mark.parametrize("variant", ["bf16", "fp8", "precision_map"])
def test_psnr_drop_and_bpp_within_north_star_gates(fp32_run, variant, tmp_path):
    x, x_ref, y_ref, med = fp32_run["x"], fp32_run["x_ref"], fp32_run["y_ref"], fp32_run["med"]
    fast = _variant(fp32_run, variant, tmp_path)
    with torch.inference_mode():
        out = fast.compress(x)
        x_hat = fast.decompress(out["strings"], out["shape"])["x_hat"]
        y = fast.model.g_a(x).float()
    torch.cuda.synchronize()
    sym_ref = torch.round(y_ref - med)
    spread = float(sym_ref.std())
    assert spread > 3.0, spread  # the latent really spans the tables
    mismatch = float((torch.round(y - med) != sym_ref).float().mean())
    y_err = float((y - y_ref).abs().max() / (y_ref.max() - y_ref.min()))
    drop = _psnr(x_ref, x) - _psnr(x_hat, x)
    bpp_ratio = out["strings"][0].packed.numel() / fp32_run["bytes"]
    close = _psnr(x_hat, x_ref)
    print(f"\n{variant}: symbol mismatch {mismatch:.4%}, max latent error {y_err:.4%} of its range, "
          f"PSNR drop {drop:.5f} dB, bpp ratio {bpp_ratio:.5f}, PSNR vs FP32 reconstruction {close:.2f} dB")
    assert drop <= 0.1, drop
    assert abs(bpp_ratio - 1.0) <= 0.01, bpp_ratio
    # bounds of the arithmetic: bf16 operands and activations keep the latent
    # within 1% of its range; e4m3 operands (3 mantissa bits) within 5%,
    # which at this spread is about half a quantisation step, so about half
    # of the symbols move by one while the gates above still hold
    assert y_err < (0.01 if variant == "bf16" else 0.05), y_err
    assert mismatch < (0.05 if variant == "bf16" else 0.75), mismatch
    assert close > (35.0 if variant == "bf16" else 25.0), close
