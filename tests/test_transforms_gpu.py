"""GPU tests of the tcgen05 transform layers (include/fcai_transforms.h).

Per layer, the kernel is compared with a PyTorch fp32 computation of the
same arithmetic: bf16-rounded input and weights, fp32 accumulation, bias,
GDN on bf16(x^2) with bf16 gamma, bf16 output.  Tolerance: 1% of each value
plus 0.1% of the tensor's max magnitude (bf16 output rounding is 0.4%; the
rest covers fp32 summation order and approximate rsqrt).
The whole g_a / g_s pair is then compared with the FP32 model.
"""

from __future__ import annotations

import copy

import pytest
import torch
import torch.nn.functional as F

from fast_compressai import accelerate
from fast_compressai.balle import GDN, FactorizedPrior
from fast_compressai.coders.errors import CoderInputError
from fast_compressai.transforms import (
    FCAI_FMT_NHWC_BF16,
    B200Analysis,
    B200Synthesis,
    _make_layer,
    _run,
)

pytestmark = pytest.mark.gpu


def _bf(t):
    return t.to(torch.bfloat16).float()


def _ref_layer(x_nchw, conv, gdn, out_bf16=True, clamp=False):
    xb = _bf(x_nchw)
    wb = _bf(conv.weight)
    if isinstance(conv, torch.nn.ConvTranspose2d):
        acc = F.conv_transpose2d(xb, wb, conv.bias.float(), stride=2, padding=2, output_padding=1)
    else:
        acc = F.conv2d(xb, wb, conv.bias.float(), stride=2, padding=2)
    if gdn is not None:
        beta, gamma = gdn.effective_params()
        c = beta.numel()
        norm = F.conv2d(_bf(acc * acc), _bf(gamma).reshape(c, c, 1, 1), beta.float())
        acc = acc * (torch.sqrt(norm) if gdn.inverse else torch.rsqrt(norm))
    if clamp:
        acc = acc.clamp(0, 1)
    return _bf(acc) if out_bf16 else acc


def _check(mine, ref):
    err = (mine - ref).abs()
    bound = 0.01 * ref.abs() + 1e-3 * ref.abs().max()
    assert bool((err <= bound).all()), f"max err {err.max().item():.4g} vs ref max {ref.abs().max().item():.4g}"


def _nhwc(x):
    return x.permute(0, 2, 3, 1).contiguous().to(torch.bfloat16)


# widths divisible by 4 take the TMA input-window path (tiles of up to 64
# columns; 260 -> 130 output columns is ragged, 16 -> tiles 8 wide and 16
# high), the others the direct-load path
@pytest.mark.parametrize("H,W", [(64, 96), (40, 72), (36, 260), (16, 16), (33, 47)])
def test_first_layer_gather_gdn(cuda_device, H, W):
    torch.manual_seed(1)
    conv = torch.nn.Conv2d(3, 128, 5, 2, 2).to(cuda_device)
    gdn = GDN(128).to(cuda_device)
    with torch.no_grad():
        gdn.gamma.add_(torch.rand_like(gdn.gamma) * 0.05)
        x = torch.rand(2, 3, H, W, device=cuda_device)
        layer = _make_layer(conv, gdn, first=True, out_f32=False, clamp=False)
        out = _run([layer], x, first_is_nchw=True)
        torch.cuda.synchronize()
        mine = out.float().permute(0, 3, 1, 2)
        _check(mine, _ref_layer(x, conv, gdn))


# pair=True: CTA pairs (2-SM MMAs), the algorithm for 128 / 192 output
# channels that callers can ask for; pair=False: one CTA per 128-pixel tile
@pytest.mark.parametrize("pair", [False, True])
@pytest.mark.parametrize("cin,cout,use_gdn,H,W", [(128, 128, True, 64, 96), (128, 128, True, 37, 50),
                                                 (128, 192, False, 32, 48), (192, 128, False, 16, 24),
                                                 (128, 128, False, 9, 70), (128, 128, True, 2, 3)])
def test_conv_layers(cuda_device, cin, cout, use_gdn, H, W, pair):
    torch.manual_seed(2)
    conv = torch.nn.Conv2d(cin, cout, 5, 2, 2).to(cuda_device)
    gdn = GDN(cout).to(cuda_device) if use_gdn else None
    with torch.no_grad():
        x = torch.randn(2, cin, H, W, device=cuda_device)
        out_f32 = not use_gdn and cout == 192
        layer = _make_layer(conv, gdn, first=False, out_f32=out_f32, clamp=False, pair=pair)
        out = _run([layer], _nhwc(x), first_is_nchw=False)
        torch.cuda.synchronize()
        mine = out if out_f32 else out.float().permute(0, 3, 1, 2)
        _check(mine, _ref_layer(x, conv, gdn, out_bf16=not out_f32))


@pytest.mark.parametrize("pair", [False, True])
@pytest.mark.parametrize("cin,cout,use_gdn,H,W", [(192, 128, True, 8, 12), (128, 128, True, 16, 24),
                                                 (128, 128, True, 9, 13), (128, 3, False, 16, 24),
                                                 (128, 3, False, 9, 13), (128, 3, False, 31, 47)])
def test_deconv_layers(cuda_device, cin, cout, use_gdn, H, W, pair):
    torch.manual_seed(3)
    deconv = torch.nn.ConvTranspose2d(cin, cout, 5, 2, 2, output_padding=1).to(cuda_device)
    gdn = GDN(cout, inverse=True).to(cuda_device) if use_gdn else None
    with torch.no_grad():
        x = torch.randn(2, cin, H, W, device=cuda_device) * 0.5
        out_f32 = cout == 3
        for clamp in ((False, True) if out_f32 else (False,)):
            layer = _make_layer(deconv, gdn, first=False, out_f32=out_f32, clamp=clamp, pair=pair and cout > 10)
            out = _run([layer], _nhwc(x), first_is_nchw=False)
            torch.cuda.synchronize()
            mine = out if out_f32 else out.float().permute(0, 3, 1, 2)
            assert mine.shape == (2, cout, 2 * H, 2 * W)
            _check(mine, _ref_layer(x, deconv, gdn, out_bf16=not out_f32, clamp=clamp))


def _psnr(a, b):
    mse = ((a - b) ** 2).mean().item()
    return 10 * torch.log10(torch.tensor(1.0 / max(mse, 1e-20))).item()


def _smooth_images(B, H, W, device, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(B, 3, H, W, generator=g)
    x = F.avg_pool2d(F.pad(x, (2, 2, 2, 2), mode="reflect"), 5, stride=1)
    lo = x.amin(dim=(1, 2, 3), keepdim=True)
    hi = x.amax(dim=(1, 2, 3), keepdim=True)
    return ((x - lo) / (hi - lo)).to(device)


def test_full_transforms_against_fp32(cuda_device):
    torch.manual_seed(0)
    model = FactorizedPrior(128, 192).to(cuda_device).eval()
    x = _smooth_images(2, 128, 192, cuda_device)
    with torch.no_grad():
        y_ref = model.g_a(x)
        ga = B200Analysis(model.g_a)
        gs = B200Synthesis(model.g_s)
        y = ga(x)
        assert y.shape == y_ref.shape and y.dtype == torch.float32
        rel = (y - y_ref).abs().max() / y_ref.abs().max()
        # the same model in PyTorch bf16 (the reference's BF16 candidates)
        y_bf = copy.deepcopy(model.g_a).to(torch.bfloat16)(x.to(torch.bfloat16)).float()
        rel_bf = (y_bf - y_ref).abs().max() / y_ref.abs().max()
        assert rel < max(2 * rel_bf, 0.02), (rel.item(), rel_bf.item())
        x_ref = model.g_s(y_ref)
        x_mine = gs(y_ref)
        assert x_mine.shape == x.shape
        rel_s = (x_mine - x_ref).abs().max() / x_ref.abs().max()
        assert rel_s < 0.05, rel_s.item()
        clamped = gs(y_ref, clamp=True)
        assert torch.equal(clamped, x_mine.clamp(0, 1))
    torch.cuda.synchronize()


def test_accelerate_bf16_end_to_end(cuda_device):
    torch.manual_seed(0)
    model = FactorizedPrior(128, 192).to(cuda_device).eval()
    model.update(force=True)
    x = _smooth_images(2, 128, 192, cuda_device, seed=3)
    fast = accelerate(model, P=4, device="cuda:0", transforms="bf16")
    assert fast.acceleration_report.runtime_status == "applied"
    assert set(fast.state_dict()) == set(model.state_dict())
    with torch.inference_mode():
        out = fast.compress(x)
        x_hat = fast.decompress(out["strings"], out["shape"])["x_hat"]
        eb = model.entropy_bottleneck
        med = eb._get_medians().detach().reshape(1, -1, 1, 1)
        y_ref = model.g_a(x)
        x_ref = model.g_s(torch.round(y_ref - med) + med).clamp(0, 1)
        # decoded symbols are exactly the quantised B200 latent
        y_fast = fast.model.g_a(x)
        sym_fast = torch.round(y_fast - med).int()
        fe = fast.model.entropy_bottleneck
        idx = fe._build_indexes(sym_fast.shape, device="cuda:0").reshape(2, -1).contiguous()
        dec = fast._coder.backend.decode(out["strings"][0], idx, fe._quantized_cdf.contiguous(),
                                         fe._cdf_length.contiguous(), fe._offset.contiguous())
    assert torch.equal(dec.reshape_as(sym_fast), sym_fast)
    assert x_hat.shape == x.shape and float(x_hat.min()) >= 0 and float(x_hat.max()) <= 1
    # the bf16 pipeline stays close to the fp32 reference reconstruction, and
    # its PSNR against the input drops by at most 0.1 dB
    assert _psnr(x_hat, x_ref) > 25.0, _psnr(x_hat, x_ref)
    drop = _psnr(x_ref, x) - _psnr(x_hat, x)
    assert drop <= 0.1, drop
    # and its payload stays within 1% of the FP32 path's (bpp gate)
    ref_fast = accelerate(model, P=4, device="cuda:0", transforms="fp32")
    with torch.inference_mode():
        ref_bytes = ref_fast.compress(x)["strings"][0].packed.numel()
    assert abs(out["strings"][0].packed.numel() / ref_bytes - 1.0) <= 0.01


@pytest.mark.parametrize("B,H,W", [(1, 16, 16), (2, 40, 56), (1, 17, 33)])
def test_bf16_codec_at_tiny_and_ragged_sizes(cuda_device, B, H, W):
    # a 1 x 1 latent, and sizes that are not multiples of 16 (the latent is
    # ceil-halved four times; the reconstruction is 16 x the latent): the
    # decoded symbols are the quantised B200 latent bit for bit, and
    # decompress is the B200 synthesis of exactly them
    torch.manual_seed(0)
    model = FactorizedPrior(128, 192).to(cuda_device).eval()
    model.update(force=True)
    fast = accelerate(model, P=4, device="cuda:0", transforms="bf16")
    x = _smooth_images(B, H, W, cuda_device, seed=H + W)
    with torch.inference_mode():
        out = fast.compress(x)
        x_hat = fast.decompress(out["strings"], out["shape"])["x_hat"]
        fe = fast.model.entropy_bottleneck
        med = fe._get_medians().detach().reshape(1, -1, 1, 1)
        y = fast.model.g_a(x)
        sym = torch.round(y - med).int()
        assert out["shape"] == tuple(y.shape[-2:])
        idx = fe._build_indexes(sym.shape, device="cuda:0").reshape(B, -1).contiguous()
        dec = fast._coder.backend.decode(out["strings"][0], idx, fe._quantized_cdf.contiguous(),
                                         fe._cdf_length.contiguous(), fe._offset.contiguous())
        expect = fast.model.g_s(sym.float() + med, clamp=True)
    assert torch.equal(dec.reshape_as(sym), sym)
    assert x_hat.shape == (B, 3, 16 * y.shape[-2], 16 * y.shape[-1])
    assert torch.equal(x_hat, expect)


@pytest.mark.parametrize("transforms", ["bf16", "fp32"])
def test_host_batch_entry_points_match_device_ones(cuda_device, transforms):
    # compress_host / decompress_host overlap the PCIe copies with the
    # transforms chunk by chunk (ragged last chunk included).  The B200
    # kernels compute every image the same way whatever the batch, so with
    # bf16 transforms payload and reconstruction are those of compress /
    # decompress on the device bit for bit; cuDNN (fp32) may pick another
    # algorithm for a smaller batch, so there they agree within rounding.
    torch.manual_seed(0)
    model = FactorizedPrior(128, 192).to(cuda_device).eval()
    model.update(force=True)
    x = _smooth_images(5, 64, 96, "cpu", seed=7).pin_memory()
    fast = accelerate(model, P=4, device="cuda:0", transforms=transforms)
    exact = transforms == "bf16"
    with torch.inference_mode():
        ref = fast.compress(x.to(cuda_device))
        x_ref = fast.decompress(ref["strings"], ref["shape"])["x_hat"]
        out = fast.compress_host(x, chunk_images=2)
        assert out["shape"] == ref["shape"]
        if exact:
            assert torch.equal(out["strings"][0].packed, ref["strings"][0].packed)
        x_dev = fast.decompress(out["strings"], out["shape"])["x_hat"]
        host = torch.empty(x_ref.shape, dtype=x_ref.dtype).pin_memory()
        res = fast.decompress_host(out["strings"], out["shape"], host, chunk_images=2)
        torch.cuda.synchronize()
        assert res["x_hat"] is host
        fresh = fast.decompress_host(out["strings"], out["shape"], chunk_images=3)["x_hat"]
        torch.cuda.synchronize()
        assert fresh.device.type == "cpu"
        for got in (host, fresh):
            if exact:
                assert torch.equal(got, x_dev.cpu()) and torch.equal(got, x_ref.cpu())
            else:
                torch.testing.assert_close(got, x_dev.cpu(), atol=1e-4, rtol=0)
    with pytest.raises(CoderInputError):
        fast.compress_host(x.to(cuda_device))


def test_streamed_host_batches_match_device_ones(cuda_device):
    # upload_host starts a batch's upload on the upload stream, compress waits
    # for that upload alone, and decompress_host(ordered=False) leaves the
    # download on the download stream with a "ready" event: with three
    # batches in flight, every payload and reconstruction equals the device
    # path's bit for bit
    torch.manual_seed(0)
    model = FactorizedPrior(128, 192).to(cuda_device).eval()
    model.update(force=True)
    fast = accelerate(model, P=4, device="cuda:0", transforms="bf16")
    xs = [_smooth_images(3, 64, 96, "cpu", seed=s).pin_memory() for s in (11, 12, 13)]
    outs = [torch.empty(x.shape, dtype=torch.float32).pin_memory() for x in xs]
    with torch.inference_mode():
        refs = [fast.compress(x.to(cuda_device)) for x in xs]
        x_refs = [fast.decompress(r["strings"], r["shape"])["x_hat"].cpu() for r in refs]
        torch.cuda.synchronize()
        ups = [fast.upload_host(x) for x in xs]
        readies = []
        for up, ref, out in zip(ups, refs, outs):
            got = fast.compress(up)
            assert got["shape"] == ref["shape"]
            assert torch.equal(got["strings"][0].packed, ref["strings"][0].packed)
            res = fast.decompress_host(got["strings"], got["shape"], out, chunk_images=2, ordered=False)
            assert res["x_hat"] is out
            readies.append(res["ready"])
        for ev, out, x_ref in zip(readies, outs, x_refs):
            ev.synchronize()
            assert torch.equal(out, x_ref)
    with pytest.raises(CoderInputError):
        fast.upload_host(xs[0].to(cuda_device))


@pytest.mark.parametrize("kind", ["conv_gdn", "deconv_igdn", "conv_latent"])
def test_pair_tiles_match_single_tiles_bitwise(cuda_device, kind):
    # FCAI_ALGO_IMPLICIT_GEMM_PAIR accumulates the same products in the same
    # order as the one-CTA algorithm, so the outputs are identical
    torch.manual_seed(5)
    if kind == "conv_gdn":
        mod, gdn, shape, f32 = torch.nn.Conv2d(128, 128, 5, 2, 2), GDN(128), (3, 45, 71, 128), False
    elif kind == "deconv_igdn":
        mod, gdn = torch.nn.ConvTranspose2d(128, 128, 5, 2, 2, output_padding=1), GDN(128, inverse=True)
        shape, f32 = (3, 19, 27, 128), False
    else:
        mod, gdn, shape, f32 = torch.nn.Conv2d(128, 192, 5, 2, 2), None, (2, 30, 50, 128), True
    mod = mod.to(cuda_device)
    gdn = gdn.to(cuda_device) if gdn is not None else None
    with torch.no_grad():
        x = torch.randn(*shape, device=cuda_device).to(torch.bfloat16)
        outs = [_run([_make_layer(mod, gdn, first=False, out_f32=f32, clamp=False, pair=pr)], x, first_is_nchw=False)
                for pr in (False, True)]
        torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
