"""compress_async: the encode split into submit and finish, for overlapped
batches (the reference's execution_mode="overlap").  The payload equals the
synchronous compress's byte for byte; an overlapped loop (batch k+1's g_a
and encode enqueued before batch k's decode and g_s) reconstructs every batch
as the serial loop does; the encode runs on an encode stream of the
compute stream, and work enqueued on the compute stream after result()
sees the payload however late the pack runs; a second submit on a stream
before the finish is refused; a staging overflow at the finish falls back to
the synchronous encode with the workspace it needs."""

from __future__ import annotations

import pytest
import torch

from fast_compressai import accelerate
from fast_compressai.balle import FactorizedPrior
from fast_compressai.coders import _warp_div as ext
from fast_compressai.coders.errors import CoderError
from fast_compressai.coders.factorized import _copy_stream
from tests.test_transforms_gpu import _smooth_images

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def fast(cuda_device):
    torch.manual_seed(0)
    model = FactorizedPrior(128, 192).to(cuda_device).eval()
    model.update(force=True)
    return accelerate(model, P=4, device="cuda:0", transforms="bf16")


def test_async_payload_equals_sync(fast, cuda_device):
    x = _smooth_images(3, 128, 192, cuda_device, seed=1)
    with torch.inference_mode():
        a = fast.compress(x)["strings"][0]
        pending = fast.compress_async(x)
        out = pending.result()
        assert pending.result() is out
        b = out["strings"][0]
    torch.cuda.synchronize()
    assert torch.equal(a.packed, b.packed) and torch.equal(a.max_rounds, b.max_rounds)
    assert out["shape"] == (8, 12)


def test_overlapped_loop_matches_serial(fast, cuda_device):
    xs = [_smooth_images(2, 128, 192, cuda_device, seed=10 + i) for i in range(3)]
    with torch.inference_mode():
        serial = []
        for x in xs:
            o = fast.compress(x)
            serial.append((o["strings"][0].packed.clone(), fast.decompress(o["strings"], o["shape"])["x_hat"]))
        got = []
        pending = fast.compress_async(xs[0])
        for k in range(len(xs)):
            o = pending.result()
            if k + 1 < len(xs):
                pending = fast.compress_async(xs[k + 1])  # enqueued before this batch's decode
            got.append((o["strings"][0].packed, fast.decompress(o["strings"], o["shape"])["x_hat"]))
    torch.cuda.synchronize()
    for (pa, xa), (pb, xb) in zip(serial, got):
        assert torch.equal(pa, pb) and torch.equal(xa, xb)


def test_one_pending_encode_per_stream(fast, cuda_device):
    # the pending encode lives on the compute stream's encode stream: a
    # synchronous compress on the compute stream runs beside it, a second
    # compress_async waits for the first one's result()
    x = _smooth_images(1, 64, 64, cuda_device, seed=3)
    with torch.inference_mode():
        pending = fast.compress_async(x)
        sync = fast.compress(x)["strings"][0]
        with pytest.raises(CoderError, match="awaits fcai_warp_div_encode_finish"):
            fast.compress_async(x)
        got = pending.result()["strings"][0]
        again = fast.compress_async(x).result()["strings"][0]  # the encode stream is free again
    torch.cuda.synchronize()
    assert torch.equal(sync.packed, got.packed) and torch.equal(got.packed, again.packed)


def test_staging_overflow_falls_back_to_the_synchronous_encode(cuda_device):
    # latents far outside the CDF range: every symbol escapes with several
    # nibbles, more staged words than the first workspace holds
    torch.manual_seed(2)
    C, HW, B = 16, 64, 2
    L = 12
    pmf = torch.rand(C, L - 1) + 0.1
    cdf = torch.zeros(C, L, dtype=torch.int64)
    cdf[:, 1:] = torch.cumsum(pmf / pmf.sum(1, keepdim=True) * 65535, 1).round().long()
    cdf[:, -1] = 65536
    for c in range(C):
        for i in range(1, L):
            cdf[c, i] = max(int(cdf[c, i]), int(cdf[c, i - 1]) + 1)
        cdf[c, -1] = 65536
    cdfs = cdf.to(torch.int32).to(cuda_device)
    sizes = torch.full((C,), L, dtype=torch.int32, device=cuda_device)
    offs = torch.full((C,), -5, dtype=torch.int32, device=cuda_device)
    med = torch.zeros(C, device=cuda_device)
    y = (torch.randn(B, C, 8, 8, device=cuda_device) * 1e7).contiguous()
    sync = ext.encode_latent(y, med, cdfs, sizes, offs, 4)
    ext.release_workspaces()  # the submit sizes its first workspace afresh
    pending = ext.encode_latent_submit(y, med, cdfs, sizes, offs, 4)
    got = ext.encode_finish(pending)
    torch.cuda.synchronize()
    assert torch.equal(sync.packed, got.packed) and torch.equal(sync.max_rounds, got.max_rounds)
    assert got.packed.numel() > B * C * HW * 4  # more than one word per symbol: the overflow path ran
    with pytest.raises(RuntimeError, match="already finished"):
        ext.encode_finish(pending)


def test_finish_waits_for_the_encode_only(fast, cuda_device):
    # work enqueued after the submit (a long sleep) does not delay the finish
    x = _smooth_images(1, 64, 64, cuda_device, seed=4)
    with torch.inference_mode():
        pending = fast.compress_async(x)
        torch.cuda._sleep(2_000_000_000)  # about a second of device time after the encode
        out = pending.result()
        assert not torch.cuda.current_stream().query()  # the sleep is still running
    torch.cuda.synchronize()
    assert out["strings"][0].packed.numel() > 0


def test_compute_stream_waits_for_a_late_pack(fast, cuda_device):
    # the pack queued behind a long sleep on the encode stream: a read of the
    # payload on the compute stream right after result() still sees it whole
    x = _smooth_images(2, 64, 64, cuda_device, seed=5)
    with torch.inference_mode():
        sync = fast.compress(x)["strings"][0]
        compute = torch.cuda.current_stream()
        encode = _copy_stream(compute.device, compute, "encode")
        pending = fast.compress_async(x)
        with torch.cuda.stream(encode):
            torch.cuda._sleep(500_000_000)  # enqueued after the encode, before the pack
        got = pending.result()["strings"][0]
        same = torch.equal(got.packed, sync.packed) and torch.equal(got.max_rounds, sync.max_rounds)
    assert same
