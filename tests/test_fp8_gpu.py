"""FP8 (e4m3) transform layers and saved precision maps on the B200.

The quantiser is compared with the reference's rule bit for bit
(backends/pytorch/fp8_operators.py:44-51: scale = max(amax / 448, FLT_MIN),
q = e4m3(clamp(x / scale, +-448))).  The e4m3 layers are compared with a
torch emulation of the same scaled GEMM: dequantised e4m3 operands, fp32
convolution, scale, bias, then GDN / IGDN with bf16 x^2 and gamma; the
tolerance covers the accumulation order and the bf16 output rounding.
"""

from __future__ import annotations

import ctypes
import json
from pathlib import Path

import pytest
import torch
import torch.nn.functional as F

from fast_compressai import _native, accelerate
from fast_compressai.balle import GDN, FactorizedPrior
from fast_compressai.configs import PrecisionConfig, model_fingerprint
from fast_compressai.transforms import FP8_MAX, FP8_SCALE_MIN, _make_layer, _run

pytestmark = pytest.mark.gpu
FIXTURE = Path(__file__).parent / "golden" / "precision_map_factorized.json"


def _bf(t):
    return t.to(torch.bfloat16).float()


def _ref_quant(x):
    scale = torch.clamp(x.float().abs().amax() / FP8_MAX, min=FP8_SCALE_MIN)
    return torch.clamp(x.float() / scale, -FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn), scale


def _quantize(x_bf16):
    q = torch.empty(x_bf16.shape, dtype=torch.uint8, device=x_bf16.device)
    scal = torch.empty(2, dtype=torch.float32, device=x_bf16.device)
    stream = torch.cuda.current_stream().cuda_stream
    _native.check(_native.lib().fcai_quantize_e4m3(ctypes.c_void_p(x_bf16.data_ptr()), ctypes.c_void_p(q.data_ptr()),
                                                   ctypes.c_void_p(scal.data_ptr()),
                                                   ctypes.c_void_p(scal.data_ptr() + 4), 0, x_bf16.numel(),
                                                   ctypes.c_void_p(stream)))
    return q, scal[0]


@pytest.mark.parametrize("shape,spread", [((4, 16, 24, 128), 1.0), ((2, 5, 7, 64), 300.0), ((1, 1, 1, 8), 1e-30)])
def test_quantiser_matches_the_reference_rule(cuda_device, shape, spread):
    torch.manual_seed(0)
    x = (torch.randn(shape, device=cuda_device) * spread).to(torch.bfloat16)
    q, scale = _quantize(x)
    ref_q, ref_scale = _ref_quant(x)
    torch.cuda.synchronize()
    assert scale.item() == ref_scale.item()
    assert torch.equal(q, ref_q.view(torch.uint8))
    zeros = torch.zeros(64, dtype=torch.bfloat16, device=cuda_device)
    qz, sz = _quantize(zeros)
    assert sz.item() == FP8_SCALE_MIN and int(qz.abs().sum()) == 0


@pytest.mark.parametrize("amax", [1.0, 300.0, 1e-30, 3.0e38, 0.0])
def test_quantiser_every_bf16_pattern(cuda_device, amax):
    # all 65536 bf16 bit patterns (zeros, subnormals, infinities and NaNs
    # included) through the quantiser with a given amax, against the
    # reference's rule evaluated by torch with the scale the call wrote
    x = torch.arange(65536, dtype=torch.int32, device=cuda_device).to(torch.int16).view(torch.bfloat16)
    q = torch.empty(65536, dtype=torch.uint8, device=cuda_device)
    scal = torch.tensor([0.0, amax], dtype=torch.float32, device=cuda_device)
    stream = torch.cuda.current_stream().cuda_stream
    _native.check(_native.lib().fcai_quantize_e4m3(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(q.data_ptr()),
                                                   ctypes.c_void_p(scal.data_ptr()),
                                                   ctypes.c_void_p(scal.data_ptr() + 4), 1, 65536,
                                                   ctypes.c_void_p(stream)))
    torch.cuda.synchronize()
    scale = scal[0:1]
    assert scale.item() == max(float(torch.tensor(amax, dtype=torch.float32) * torch.tensor(1.0 / 448.0)),
                               FP8_SCALE_MIN)
    ref = torch.clamp(x.float() / scale, -FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn).view(torch.uint8)
    assert torch.equal(q, ref), f"{int((q != ref).sum())} patterns differ"


def _ref_fp8_layer(x_nchw, conv, gdn, out_bf16=True):
    """The scaled GEMM on dequantised e4m3 operands, then bias and (I)GDN."""
    xq, xs = _ref_quant(_bf(x_nchw))
    wq, ws = _ref_quant(conv.weight)
    xd = xq.float() * xs
    wd = wq.float() * ws
    if isinstance(conv, torch.nn.ConvTranspose2d):
        acc = F.conv_transpose2d(xd, wd, conv.bias.float(), stride=2, padding=2, output_padding=1)
    else:
        acc = F.conv2d(xd, wd, conv.bias.float(), stride=2, padding=2)
    if gdn is not None:
        beta, gamma = gdn.effective_params()
        c = beta.numel()
        norm = F.conv2d(_bf(acc * acc), _bf(gamma).reshape(c, c, 1, 1), beta.float())
        acc = acc * (torch.sqrt(norm) if gdn.inverse else torch.rsqrt(norm))
    return _bf(acc) if out_bf16 else acc


def _check(mine, ref):
    err = (mine - ref).abs()
    bound = 0.02 * ref.abs() + 4e-3 * ref.abs().max()
    assert bool((err <= bound).all()), f"max err {err.max().item():.4g} vs ref max {ref.abs().max().item():.4g}"


@pytest.mark.parametrize("kind,cout,use_gdn,H,W", [("conv", 128, True, 32, 48), ("conv", 128, True, 9, 13),
                                                  ("conv", 192, False, 16, 24), ("deconv", 128, True, 16, 24),
                                                  ("conv", 128, False, 8, 40)])
def test_fp8_layers_match_the_scaled_gemm(cuda_device, kind, cout, use_gdn, H, W):
    torch.manual_seed(4)
    if kind == "conv":
        conv = torch.nn.Conv2d(128, cout, 5, 2, 2).to(cuda_device)
    else:
        conv = torch.nn.ConvTranspose2d(128, cout, 5, 2, 2, output_padding=1).to(cuda_device)
    gdn = GDN(cout, inverse=kind == "deconv").to(cuda_device) if use_gdn else None
    with torch.no_grad():
        x = torch.randn(2, 128, H, W, device=cuda_device)
        out_f32 = cout == 192
        layer = _make_layer(conv, gdn, first=False, out_f32=out_f32, clamp=False, precision="fp8")
        out = _run([layer], x.permute(0, 2, 3, 1).contiguous().to(torch.bfloat16), first_is_nchw=False)
        torch.cuda.synchronize()
        mine = out if out_f32 else out.float().permute(0, 3, 1, 2)
        _check(mine, _ref_fp8_layer(x, conv, gdn, out_bf16=not out_f32))


@pytest.mark.parametrize("kind", ["conv_gdn", "deconv_igdn", "first_layer"])
def test_producer_amax_equals_the_tensor_amax(cuda_device, kind):
    # a layer whose output feeds an FP8 layer reports max |output| over its
    # valid pixels (ragged tiles included) through amax_out; the quantiser
    # then skips its own pass.  Bit-exact with the amax of the output tensor.
    torch.manual_seed(5)
    first = kind == "first_layer"
    if kind == "deconv_igdn":
        conv = torch.nn.ConvTranspose2d(128, 128, 5, 2, 2, output_padding=1).to(cuda_device)
        gdn = GDN(128, inverse=True).to(cuda_device)
        x = torch.randn(2, 128, 9, 13, device=cuda_device)
    elif first:
        conv = torch.nn.Conv2d(3, 128, 5, 2, 2).to(cuda_device)
        gdn = GDN(128).to(cuda_device)
        x = torch.rand(2, 3, 36, 52, device=cuda_device)
    else:
        conv = torch.nn.Conv2d(128, 128, 5, 2, 2).to(cuda_device)
        gdn = GDN(128).to(cuda_device)
        x = torch.randn(2, 128, 37, 50, device=cuda_device)
    nxt = torch.nn.Conv2d(128, 128, 5, 2, 2).to(cuda_device)
    with torch.no_grad():
        a = _make_layer(conv, gdn, first=first, out_f32=False, clamp=False)
        b = _make_layer(nxt, GDN(128).to(cuda_device), first=False, out_f32=False, clamp=False, precision="fp8")
        inp = x if first else x.permute(0, 2, 3, 1).contiguous().to(torch.bfloat16)
        mid = _run([a], inp, first_is_nchw=first)
        both = _run([a, b], inp, first_is_nchw=first)  # amax from a's epilogue
        alone = _run([b], mid, first_is_nchw=False)      # amax pass of the quantiser
        torch.cuda.synchronize()
        assert torch.equal(both, alone)
        assert a.desc.amax_out is None


def _map_for(model, p_ch, tmp_path):
    data = json.loads(FIXTURE.read_text())
    data["model_fingerprint"] = model_fingerprint(model)
    data["p_ch"] = p_ch
    path = tmp_path / "map.json"
    path.write_text(json.dumps(data))
    return path


def test_precision_map_through_accelerate(cuda_device, tmp_path):
    # the reference's example map: g_a.2 and g_a.6 run the e4m3 kernels, the
    # rest bf16; compress / decompress round-trip and stay close to FP32
    torch.manual_seed(0)
    model = FactorizedPrior(128, 192).to(cuda_device).eval()
    model.update(force=True)
    path = _map_for(model, 4, tmp_path)
    fast = accelerate(model, P=4, device="cuda:0", precision_config_path=str(path))
    report = fast.acceleration_report
    assert report.precision_selection_status == "loaded_from_config"
    applied = {p: (want, got) for p, want, got, _ in report.precision_applications}
    assert applied["g_a.2"] == ("fp8", "fp8") and applied["g_a.6"] == ("fp8", "fp8")
    assert applied["g_a.0"] == ("fp16", "bf16") and applied["g_s.1"] == ("fp8", "bf16")
    ref = accelerate(model, P=4, device="cuda:0")  # FP32 transforms
    g = torch.Generator().manual_seed(3)
    x = F.avg_pool2d(torch.rand(2, 3, 128, 192, generator=g), 5, 1, 2).to(cuda_device)
    x = (x - x.amin()) / (x.amax() - x.amin())
    with torch.inference_mode():
        out = fast.compress(x)
        x_hat = fast.decompress(out["strings"], out["shape"])["x_hat"]
        out_ref = ref.compress(x)
        x_ref = ref.decompress(out_ref["strings"], out_ref["shape"])["x_hat"]
    torch.cuda.synchronize()
    assert x_hat.shape == x.shape and bool(torch.isfinite(x_hat).all())

    def psnr(a, b):
        return float(10 * torch.log10(1.0 / F.mse_loss(a.float(), b.float())))

    # the north star's gates (the same gates on latents that span the CDF
    # tables: tests/test_quality_gpu.py)
    assert psnr(x_ref, x) - psnr(x_hat, x) <= 0.1
    bpp = out["strings"][0].packed.numel() / out_ref["strings"][0].packed.numel()
    assert abs(bpp - 1.0) <= 0.01
    with pytest.raises(Exception, match="model fingerprint"):
        other = FactorizedPrior(128, 192).to(cuda_device)
        accelerate(other, P=4, device="cuda:0", precision_config_path=str(path))
    with pytest.raises(Exception, match="coder/P_ch"):
        accelerate(model, P=8, device="cuda:0", precision_config_path=str(path))
