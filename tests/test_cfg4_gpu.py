"""BASELINE config 4 shapes on the B200 kernels: FactorizedPrior(N=192,
M=320).  GDN / IGDN over 192 channels (one TMEM accumulator buffer: the
accumulator and the norm fill it), the 192-channel first layer, the 320 ->
192 transposed convolution and the 320-channel latent layer (two launches of
160 channels writing one fp32 output).  Per layer against a torch emulation
of the same bf16 rounding points, then the whole model against FP32
transforms: PSNR drop <= 0.1 dB, payload within 1%, and decoded symbols
equal to the quantised latent."""

from __future__ import annotations

import pytest
import torch

from fast_compressai import accelerate
from fast_compressai.balle import GDN, FactorizedPrior
from fast_compressai.transforms import _make_layer, _run
from tests.test_transforms_gpu import _check, _nhwc, _psnr, _ref_layer, _smooth_images

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind,cin,cout,H,W", [("conv_gdn", 192, 192, 32, 48), ("conv_gdn", 192, 192, 9, 13),
                                              ("deconv_igdn", 192, 192, 16, 24), ("deconv_igdn", 320, 192, 8, 12),
                                              ("latent", 192, 320, 16, 24), ("first", 3, 192, 64, 96),
                                              ("first", 3, 192, 33, 47)])
def test_config4_layers(cuda_device, kind, cin, cout, H, W):
    torch.manual_seed(6)
    first = kind == "first"
    if kind == "deconv_igdn":
        conv = torch.nn.ConvTranspose2d(cin, cout, 5, 2, 2, output_padding=1).to(cuda_device)
        gdn = GDN(cout, inverse=True).to(cuda_device)
    else:
        conv = torch.nn.Conv2d(cin, cout, 5, 2, 2).to(cuda_device)
        gdn = GDN(cout).to(cuda_device) if kind != "latent" else None
    with torch.no_grad():
        if gdn is not None:
            gdn.gamma.add_(torch.rand_like(gdn.gamma) * 0.05)
        x = torch.rand(2, cin, H, W, device=cuda_device) if first else torch.randn(2, cin, H, W, device=cuda_device)
        out_f32 = kind == "latent"
        layer = _make_layer(conv, gdn, first=first, out_f32=out_f32, clamp=False)
        assert bool(layer.parts) == (kind == "latent")
        out = _run([layer], x if first else _nhwc(x), first_is_nchw=first)
        torch.cuda.synchronize()
        mine = out if out_f32 else out.float().permute(0, 3, 1, 2)
        _check(mine, _ref_layer(x, conv, gdn, out_bf16=not out_f32))


def test_config4_model_end_to_end(cuda_device):
    torch.manual_seed(0)
    model = FactorizedPrior(192, 320).to(cuda_device).eval()
    model.update(force=True)
    x = _smooth_images(2, 128, 192, cuda_device, seed=9)
    fast = accelerate(model, P=8, device="cuda:0", transforms="bf16")
    ref = accelerate(model, P=8, device="cuda:0")
    with torch.inference_mode():
        out = fast.compress(x)
        x_hat = fast.decompress(out["strings"], out["shape"])["x_hat"]
        out_ref = ref.compress(x)
        eb = model.entropy_bottleneck
        med = eb._get_medians().detach().reshape(1, -1, 1, 1)
        x_ref = model.g_s(torch.round(model.g_a(x) - med) + med).clamp(0, 1)
        y_fast = fast.model.g_a(x)
        sym = torch.round(y_fast - med).int()
        fe = fast.model.entropy_bottleneck
        idx = fe._build_indexes(sym.shape, device="cuda:0").reshape(2, -1).contiguous()
        dec = fast._coder.backend.decode(out["strings"][0], idx, fe._quantized_cdf.contiguous(),
                                         fe._cdf_length.contiguous(), fe._offset.contiguous())
    assert torch.equal(dec.reshape_as(sym), sym)
    assert y_fast.shape == (2, 320, 8, 12)
    drop = _psnr(x_ref, x) - _psnr(x_hat, x)
    assert drop <= 0.1, drop
    ratio = out["strings"][0].packed.numel() / out_ref["strings"][0].packed.numel()
    assert abs(ratio - 1.0) <= 0.01, ratio


@pytest.mark.parametrize("kind,cin,cout,H,W", [("conv_gdn", 192, 192, 32, 48), ("conv_gdn", 192, 192, 9, 13),
                                              ("deconv_igdn", 192, 192, 16, 24), ("deconv_igdn", 320, 192, 8, 12),
                                              ("latent", 192, 320, 16, 24)])
def test_config4_fp8_layers(cuda_device, kind, cin, cout, H, W):
    # e4m3 operands with per-tensor scales; cin = 192 / 320 run K blocks of
    # 128 channels whose part past cin is zero-filled by TMA.  The split
    # latent's two launches share the whole weight's scale.
    from tests.test_fp8_gpu import _check as _check_fp8, _ref_fp8_layer

    torch.manual_seed(7)
    if kind == "deconv_igdn":
        conv = torch.nn.ConvTranspose2d(cin, cout, 5, 2, 2, output_padding=1).to(cuda_device)
        gdn = GDN(cout, inverse=True).to(cuda_device)
    else:
        conv = torch.nn.Conv2d(cin, cout, 5, 2, 2).to(cuda_device)
        gdn = GDN(cout).to(cuda_device) if kind != "latent" else None
    with torch.no_grad():
        if gdn is not None:
            gdn.gamma.add_(torch.rand_like(gdn.gamma) * 0.05)
        x = torch.randn(2, cin, H, W, device=cuda_device)
        out_f32 = kind == "latent"
        layer = _make_layer(conv, gdn, first=False, out_f32=out_f32, clamp=False, precision="fp8")
        assert layer.precision == "fp8" and bool(layer.parts) == out_f32
        if layer.parts:
            assert len({p.desc.weight_scale for p in layer.parts}) == 1
        out = _run([layer], _nhwc(x), first_is_nchw=False)
        torch.cuda.synchronize()
        mine = out if out_f32 else out.float().permute(0, 3, 1, 2)
        _check_fp8(mine, _ref_fp8_layer(x, conv, gdn, out_bf16=not out_f32))


def test_config4_model_fp8_transforms(cuda_device):
    # transforms="fp8": every convolution with an e4m3 kernel runs it (all but
    # the 3-channel first layer and the scatter layer); the model still
    # round-trips its symbols and stays close to the FP32 transforms
    torch.manual_seed(0)
    model = FactorizedPrior(192, 320).to(cuda_device).eval()
    model.update(force=True)
    x = _smooth_images(2, 128, 192, cuda_device, seed=9)
    fast = accelerate(model, P=8, device="cuda:0", transforms="fp8")
    applied = {p: got for p, _, got, _ in fast.acceleration_report.precision_applications}
    assert [applied[f"g_a.{i}"] for i in (0, 2, 4, 6)] == ["bf16", "fp8", "fp8", "fp8"]
    assert [applied[f"g_s.{i}"] for i in (0, 2, 4, 6)] == ["fp8", "fp8", "fp8", "bf16"]
    ref = accelerate(model, P=8, device="cuda:0")
    with torch.inference_mode():
        out = fast.compress(x)
        x_hat = fast.decompress(out["strings"], out["shape"])["x_hat"]
        out_ref = ref.compress(x)
        x_ref = ref.decompress(out_ref["strings"], out_ref["shape"])["x_hat"]
    assert x_hat.shape == x.shape and bool(torch.isfinite(x_hat).all())
    assert abs(_psnr(x_hat, x) - _psnr(x_ref, x)) < 1.0
    ratio = out["strings"][0].packed.numel() / out_ref["strings"][0].packed.numel()
    assert 0.9 < ratio < 1.1
