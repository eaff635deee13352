"""Bit-exact parity with the reference's own warp_div extension.

The reference extension is compiled from the reference sources for sm_100a
by oracle/build_ref.py (output oracle/_ref/_warp_div_ref.so, a test-only
checker).  Payload bytes are compared with the pad bytes between the round
table and header_bytes masked: the reference allocates the payload with
torch::empty and never writes them (warp_ans_kernel_v2.cu:280,
warp_ans_kernel.cu:343-369).  Decoders are cross-checked both ways.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from fast_compressai.coders import _warp_div as ext
from oracle import build_ref
from oracle import oracle as O
from tests.coder_inputs import channel_indexes, laplacian_symbols, laplacian_tables, small_tables

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref():
    return build_ref.load()


def _dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def _check(ref, sym, idx, cdfs, sizes, offs, P, device):
    t = [_dev(a, device) for a in (sym, idx, cdfs, sizes, offs)]
    rp, rmr, rhb, rcl, rP = ref.encode_warp_div(*t, P)
    mine = ext.encode(*t, P)
    hb = int(rhb[0])
    assert mine.header_bytes == hb and mine.chunk_len == int(rcl[0]) and int(rP[0]) == P
    assert torch.equal(mine.max_rounds, rmr)
    a, b = mine.packed.cpu().numpy(), rp.cpu().numpy()
    assert a.size == b.size
    mask = O.header_mask(a.size, hb, mine.max_rounds.numel())
    assert np.array_equal(a[mask], b[mask]), f"first diff at byte {np.argmax((a != b) & mask)}"
    # the reference decoder reads this build's payload and vice versa
    hb_t = torch.tensor([hb], dtype=torch.int64)
    cl_t = torch.tensor([mine.chunk_len], dtype=torch.int32)
    p_t = torch.tensor([P], dtype=torch.int32)
    assert torch.equal(ref.decode_warp_div(mine.packed, mine.max_rounds, hb_t, cl_t, p_t, *t[1:]), t[0])
    assert torch.equal(ext.decode_warp_div(rp, rmr, rhb, rcl, rP, *t[1:]), t[0])
    # and the CPU oracle agrees with both
    op, omr, ohb, _ = O.warp_div_encode(sym, idx, cdfs, sizes, offs, P)
    assert np.array_equal(op[mask], b[mask])


@pytest.mark.parametrize("P", [1, 2, 4])
def test_reference_known_answer_inputs(ref, cuda_device, P):
    cdfs, sizes, offs = small_tables()
    idx = np.array([[0, 1, 2, 3] * 16], dtype=np.int32)
    for sym in ([0, 1, 2, 3] * 16, [-100, 100, -101, 102] * 16):
        _check(ref, np.array([sym], dtype=np.int32), idx, cdfs, sizes, offs, P, cuda_device)


@pytest.mark.parametrize(
    "B,C,HW,P,esc",
    [(1, 12, 16, 4, 0.0), (2, 12, 16, 5, 0.02), (3, 7, 33, 3, 0.05), (1, 4, 1, 1, 0.3), (2, 192, 48, 4, 0.001),
     (2, 192, 48, 192, 0.0), (1, 320, 64, 8, 0.0), (4, 192, 1536, 4, 0.0)],
)
def test_payload_matches_reference(ref, cuda_device, B, C, HW, P, esc):
    cdfs, sizes, offs, scales = laplacian_tables(C, seed=C * 7 + P)
    sym = laplacian_symbols(B, C, HW, scales, seed=B * 31 + HW, escape_rate=esc)
    _check(ref, sym, channel_indexes(B, C, HW), cdfs, sizes, offs, P, cuda_device)


def test_arbitrary_indexes_match_reference(ref, cuda_device):
    rng = np.random.default_rng(4)
    cdfs, sizes, offs, _ = laplacian_tables(9, seed=3)
    sym = rng.integers(-45, 45, size=(2, 9 * 40)).astype(np.int32)
    idx = rng.integers(0, 9, size=(2, 9 * 40)).astype(np.int32)
    _check(ref, sym, idx, cdfs, sizes, offs, 2, cuda_device)


# BASELINE config 3 at full size: 64 x 192 x 32 x 48 Laplacian symbols, every
# P_ch of the sweep.  Encoded with NULL indexes (the channel layout, as the
# codec calls the coder) and with the explicit channel indexes the
# reference's API takes; both must give the reference's payload.
@pytest.fixture(scope="module")
def config3(cuda_device):
    B, C, HW = 64, 192, 32 * 48
    cdfs, sizes, offs, scales = laplacian_tables(C, seed=0)
    sym = laplacian_symbols(B, C, HW, scales, seed=0)
    idx = channel_indexes(B, C, HW)
    return [_dev(a, cuda_device) for a in (sym, idx, cdfs, sizes, offs)]


@pytest.mark.parametrize("P", [1, 2, 4, 8, 16, 48, 192])
def test_config3_full_size_matches_reference(ref, config3, P):
    sym, idx, cdfs, sizes, offs = config3
    rp, rmr, rhb, rcl, rP = ref.encode_warp_div(sym, idx, cdfs, sizes, offs, P)
    b = rp.cpu().numpy()
    mask = O.header_mask(b.size, int(rhb[0]), rmr.numel())
    for indexes in (None, idx):
        mine = ext.encode(sym, indexes, cdfs, sizes, offs, P)
        assert mine.header_bytes == int(rhb[0]) and mine.chunk_len == int(rcl[0])
        assert torch.equal(mine.max_rounds, rmr)
        a = mine.packed.cpu().numpy()
        assert a.size == b.size
        assert np.array_equal(a[mask], b[mask]), f"P={P}: first diff at byte {np.argmax((a != b) & mask)}"
    hb_t = torch.tensor([mine.header_bytes], dtype=torch.int64)
    cl_t = torch.tensor([mine.chunk_len], dtype=torch.int32)
    p_t = torch.tensor([P], dtype=torch.int32)
    assert torch.equal(ref.decode_warp_div(mine.packed, mine.max_rounds, hb_t, cl_t, p_t, idx, cdfs, sizes, offs), sym)
    assert torch.equal(ext.decode_warp_div(rp, rmr, rhb, rcl, rP, idx, cdfs, sizes, offs), sym)


def test_config2_model_latent_matches_reference(ref, cuda_device):
    # BASELINE config 2 (24 x 3 x 512 x 768, P = 4) through accelerate with
    # the bf16 transforms, on a model whose latent spans its CDF tables (with
    # escapes).  The fused latent encode (rounding y - median inside the
    # coder) must write the payload the reference extension writes for the
    # symbols round(y - median) and the channel indexes
    # (coders/factorized.py:46-59 of the reference).
    from fast_compressai import accelerate
    from tests.model_inputs import smooth_images, spread_latent_prior

    x = smooth_images(24, 512, 768, seed=1234, device=cuda_device)
    model = spread_latent_prior(128, 192, x[:4], target_std=12.0)
    fast = accelerate(model, P=4, device="cuda:0", transforms="bf16")
    with torch.inference_mode():
        out = fast.compress(x)
        payload = out["strings"][0]
        eb = fast.model.entropy_bottleneck
        y = fast.model.g_a(x)
        med = eb._get_medians().detach().reshape(1, -1, 1, 1)
        sym = torch.round(y - med).int()
        idx = eb._build_indexes(sym.shape, device=cuda_device).reshape(24, -1).contiguous()
        sym = sym.reshape(24, -1).contiguous()
        cdfs, sizes, offs = (t.contiguous() for t in (eb._quantized_cdf, eb._cdf_length, eb._offset))
        rp, rmr, rhb, rcl, rP = ref.encode_warp_div(sym, idx, cdfs, sizes, offs, 4)
        x_hat = fast.decompress(out["strings"], out["shape"])["x_hat"]
    vals = sym - offs.reshape(1, -1, 1).expand(24, -1, sym.shape[1] // 192).reshape(24, -1)
    maxv = (sizes - 2).reshape(1, -1, 1).expand(24, -1, sym.shape[1] // 192).reshape(24, -1)
    escapes = float(((vals < 0) | (vals >= maxv)).float().mean())
    assert 1e-4 < escapes < 0.05, escapes  # the bypass path is exercised
    assert int(sym.max()) - int(sym.min()) >= 20
    a, b = payload.packed.cpu().numpy(), rp.cpu().numpy()
    assert a.size == b.size and torch.equal(payload.max_rounds, rmr)
    mask = O.header_mask(a.size, int(rhb[0]), rmr.numel())
    assert np.array_equal(a[mask], b[mask]), f"first diff at byte {np.argmax((a != b) & mask)}"
    # and the reference decoder returns the symbols this build's decode
    # dequantised (x_hat is g_s of exactly those)
    hb_t = torch.tensor([payload.header_bytes], dtype=torch.int64)
    cl_t = torch.tensor([payload.chunk_len], dtype=torch.int32)
    dec = ref.decode_warp_div(payload.packed, payload.max_rounds, hb_t, cl_t, torch.tensor([4], dtype=torch.int32),
                              idx, cdfs, sizes, offs)
    assert torch.equal(dec, sym)
    with torch.inference_mode():
        x_ref = fast.model.g_s(dec.reshape(y.shape).float() + med).clamp(0, 1)
    assert torch.equal(x_hat, x_ref)
