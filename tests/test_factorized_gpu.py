"""End-to-end FactorizedPrior tests through ``accelerate`` (GPU).

Mirrors tests/gpu/test_factorized_gaans.py of the reference with this
package's FP32 FactorizedPrior (CompressAI is not installed): decoded
symbols equal ``quantize(g_a(x))`` bit for bit, the reconstruction equals
the FP32 path on those symbols, the source model is untouched, and bad
states / payloads are rejected with the reference's error types.
"""

from __future__ import annotations

from dataclasses import replace

import numpy as np
import pytest
import torch

from fast_compressai import accelerate
from fast_compressai.balle import FactorizedPrior
from fast_compressai.coders import WarpDivPayload
from fast_compressai.coders.errors import CoderInputError
from fast_compressai.config import ConfigurationError
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture()
def model(cuda_device):
    torch.manual_seed(20261015)
    m = FactorizedPrior(8, 12).to(cuda_device).eval()
    m.update(force=True)
    return m


@pytest.mark.parametrize("batch", [1, 2])
def test_gaans_matches_quantized_latent_for_multiple_p(model, cuda_device, batch):
    x = torch.rand(batch, 3, 64, 64, device=cuda_device)
    eb = model.entropy_bottleneck
    with torch.inference_mode():
        y = model.g_a(x)
        medians = eb._extend_ndims(eb._get_medians().detach(), 2).expand(batch, -1, -1, -1)
        expected = eb.quantize(y, "symbols", medians)
        reference = model.g_s(eb.dequantize(expected, medians, medians.dtype)).clamp_(0, 1)
    for p_ch in (1, 4, 5, 12):
        source = {k: v.clone() for k, v in model.state_dict().items()}
        fast = accelerate(model, P=p_ch, device="cuda:0")
        rep = fast.acceleration_report
        assert rep.coder_status == "warp_div" and rep.p_ch_applied and rep.runtime_status == "not_applied"
        assert next(fast.parameters()).device.type == "cuda"
        with torch.inference_mode():
            stream = fast.compress(x)
            payload = stream["strings"][0]
            assert isinstance(payload, WarpDivPayload) and payload.p_ch == p_ch
            assert stream["shape"] == (4, 4)
            recon = fast.decompress(stream["strings"], stream["shape"])["x_hat"]
            fe = fast.model.entropy_bottleneck
            idx = fe._build_indexes((batch, 12, *stream["shape"]), device="cuda:0")
            symbols = fast._coder.backend.decode(payload, idx.reshape(batch, -1).contiguous(),
                                                 fe._quantized_cdf.contiguous(), fe._cdf_length.contiguous(),
                                                 fe._offset.contiguous()).reshape_as(expected)
        assert torch.equal(expected, symbols)
        assert torch.allclose(reference, recon, atol=1e-6, rtol=1e-6)
        # payload equals the oracle's for the same symbols (bit-exact)
        ref_packed, _, _, _ = O.warp_div_encode(expected.reshape(batch, -1).cpu().numpy(), None,
                                                eb._quantized_cdf.cpu().numpy(), eb._cdf_length.cpu().numpy(),
                                                eb._offset.cpu().numpy(), p_ch)
        assert np.array_equal(payload.packed.cpu().numpy(), ref_packed)
        assert set(source) == set(fast.state_dict())
        assert all(torch.equal(v, model.state_dict()[k]) for k, v in source.items())


def test_timing_keys(model, cuda_device):
    fast = accelerate(model, P=4, device="cuda:0")
    timing: dict[str, float] = {}
    x = torch.rand(2, 3, 64, 64, device=cuda_device)
    with torch.inference_mode():
        s = fast.compress(x, timing=timing)
        fast.decompress(s["strings"], s["shape"], timing=timing)
    assert set(timing) == {"compress_inference_ms", "compress_codec_ms", "decompress_codec_ms",
                           "decompress_inference_ms"}
    assert all(v >= 0 for v in timing.values())


def test_invalid_model_state_and_metadata_are_rejected(model, cuda_device):
    fresh = FactorizedPrior(8, 12).to(cuda_device).eval()
    with pytest.raises(CoderInputError, match="update"):
        accelerate(fresh, P=4, device="cuda:0")
    with pytest.raises(CoderInputError, match="P"):
        accelerate(model, P=13, device="cuda:0")
    with pytest.raises(ConfigurationError):
        accelerate(model, P=4, device="cpu")
    fast = accelerate(model, P=4, device="cuda:0")
    with torch.inference_mode():
        stream = fast.compress(torch.rand(1, 3, 64, 64, device=cuda_device))
    payload = stream["strings"][0]
    with pytest.raises(CoderInputError):
        fast.decompress(stream["strings"], (8, 8))
    with pytest.raises(CoderInputError):
        fast.decompress([[b"cpu-rans"]], stream["shape"])
    with pytest.raises(CoderInputError, match="match"):
        fast.decompress([replace(payload, p_ch=3, chunk_len=12)], stream["shape"])
    with pytest.raises(CoderInputError, match="match"):
        fast.decompress([replace(payload, coding_fingerprint="0" * 64)], stream["shape"])
    with pytest.raises(CoderInputError, match="header"):
        corrupted = payload.packed.clone()
        corrupted[0] ^= 1
        fast.decompress([replace(payload, packed=corrupted)], stream["shape"])
    with pytest.raises(CoderInputError):
        fast.compress(torch.rand(1, 3, 64, 64))  # CPU input
