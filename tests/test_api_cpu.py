"""CPU tests of the host layer: the reference's own API tests
(tests/test_warp_div_api.py, tests/test_accelerate_api.py of the reference),
configuration rules, the coding fingerprint, and the FP32 FactorizedPrior."""

from __future__ import annotations

import hashlib
import importlib
from unittest import mock

import numpy as np
import pytest
import torch

import fast_compressai
from fast_compressai.balle import FactorizedPrior
from fast_compressai.coders import warp_div as wd
from fast_compressai.coders.errors import CoderDependencyError, CoderInputError
from fast_compressai.config import AccelerationConfig, ConfigurationError


def test_catalog_is_limited_to_two_coders():
    assert fast_compressai.coder_catalog() == ("compressai-rans", "warp_div")
    with pytest.raises(CoderDependencyError):
        fast_compressai.create_coder("compressai-rans")
    with pytest.raises(ValueError):
        fast_compressai.create_coder("nope")


def test_capability_is_lazy_and_reports_missing_extension():
    with mock.patch("fast_compressai.coders.capabilities.torch.cuda.is_available", return_value=True), \
            mock.patch("fast_compressai.coders.capabilities.importlib.util.find_spec", return_value=None):
        cap = fast_compressai.warp_div_capability("cuda:0")
    assert not cap.available and cap.backend == "warp_div" and "not built" in cap.reason


def test_capability_without_cuda():
    with mock.patch("fast_compressai.coders.capabilities.torch.cuda.is_available", return_value=False):
        cap = fast_compressai.warp_div_capability()
    assert not cap.available and "unavailable" in cap.reason


def test_backend_constructor_reports_unavailable_extension():
    with mock.patch("fast_compressai.coders.warp_div.warp_div_capability") as capability:
        capability.return_value = mock.Mock(available=False, reason="not built")
        with pytest.raises(CoderDependencyError, match="not built"):
            fast_compressai.WarpDivBackend()


def test_python_import_does_not_need_a_gpu():
    assert importlib.import_module("fast_compressai.coders.warp_div") is not None
    assert importlib.util.find_spec("fast_compressai.coders._warp_div") is not None


def test_payload_rejects_non_cuda_data():
    with pytest.raises(CoderInputError):
        fast_compressai.WarpDivPayload(packed=torch.zeros(128, dtype=torch.uint8),
                                       max_rounds=torch.zeros((1, 1), dtype=torch.uint32), header_bytes=32,
                                       chunk_len=4, p_ch=1, batch=1, symbols_per_batch=4, cdf_count=1)


def test_input_contract_rejects_wrong_dtype_before_extension():
    with pytest.raises(CoderInputError):
        wd._validate_inputs(torch.zeros((1, 4), dtype=torch.float32), torch.zeros((1, 4), dtype=torch.int32),
                            torch.tensor([[0, 65536]], dtype=torch.int32), torch.tensor([2], dtype=torch.int32),
                            torch.tensor([0], dtype=torch.int32), 1)


def test_input_contract_rejects_cpu_and_shapes():
    i32 = dict(dtype=torch.int32)
    args = (torch.zeros((1, 4), **i32), torch.zeros((1, 4), **i32), torch.tensor([[0, 65536]], **i32),
            torch.tensor([2], **i32), torch.tensor([0], **i32))
    with pytest.raises(CoderInputError, match="CUDA"):
        wd._validate_inputs(*args, 1)
    with pytest.raises(CoderInputError, match="p_ch"):
        wd._validate_inputs(*args, 0)


def test_acceleration_config_rules():
    assert AccelerationConfig.from_value({"P": 4}).p_ch == 4
    assert AccelerationConfig.from_value(None, P=3).p_ch == 3
    with pytest.raises(ConfigurationError):
        AccelerationConfig.from_value({"P": 4, "p_ch": 4})
    with pytest.raises(ConfigurationError):
        AccelerationConfig.from_value({"P": 4}, P=4)
    with pytest.raises(ConfigurationError):
        AccelerationConfig.from_value(AccelerationConfig(), P=2)
    with pytest.raises(ConfigurationError):
        AccelerationConfig(p_ch=0)
    with pytest.raises(ConfigurationError):
        AccelerationConfig(coder="zstd")
    with pytest.raises(ConfigurationError):
        AccelerationConfig(budget=float("nan"))
    with pytest.raises(ConfigurationError):
        AccelerationConfig.from_value({"bogus": 1})
    assert AccelerationConfig(budget=0.5).to_dict()["budget"] == 0.5


def test_accelerate_rejects_models_and_devices_without_gpu():
    model = FactorizedPrior(8, 12)
    with pytest.raises(TypeError):
        fast_compressai.accelerate(object())
    with pytest.raises(ConfigurationError, match="FactorizedPrior"):
        fast_compressai.accelerate(torch.nn.Linear(2, 2), P=1)
    with mock.patch("fast_compressai.api.torch.cuda.is_available", return_value=False):
        with pytest.raises(ConfigurationError, match="CUDA"):
            fast_compressai.accelerate(model, P=4)
    with mock.patch("fast_compressai.api.torch.cuda.is_available", return_value=True):
        with pytest.raises(ConfigurationError, match="device='cuda'"):
            fast_compressai.accelerate(model, P=4, device="cpu")
    wrapped = fast_compressai.accelerate(model, P=2, coder="rans")
    assert wrapped.acceleration_report.coder_status == "rans"
    assert wrapped.acceleration_report.p_ch == 2 and not wrapped.acceleration_report.p_ch_applied


def test_fingerprint_channel_cache_matches_full_digest():
    B, C, HW = 3, 5, 7
    idx = torch.arange(C, dtype=torch.int32).repeat_interleave(HW).repeat(B, 1).contiguous()
    cdfs = torch.tensor([[0, 100, 65536]] * C, dtype=torch.int32)
    sizes = torch.full((C,), 3, dtype=torch.int32)
    offs = torch.zeros(C, dtype=torch.int32)
    # the reference's formula (coders/warp_div.py:152-158)
    ref = hashlib.sha256()
    for t in (idx, cdfs, sizes, offs):
        ref.update(bytes(str(tuple(t.shape)), "ascii"))
        ref.update(t.numpy().tobytes())
    full = wd._coding_fingerprint(idx, cdfs, sizes, offs)
    cached = wd._coding_fingerprint(None, cdfs, sizes, offs, batch=B, symbols_per_batch=C * HW)
    verified = wd._coding_fingerprint(idx, cdfs, sizes, offs, channel_layout=True)
    assert full == cached == verified == ref.hexdigest()
    offs2 = offs.clone()
    offs2[0] = 1
    assert wd._coding_fingerprint(None, cdfs, sizes, offs2, batch=B, symbols_per_batch=C * HW) != full
    # in-place edits invalidate the per-tensor cache
    offs[1] = 9
    assert wd._coding_fingerprint(None, cdfs, sizes, offs, batch=B, symbols_per_batch=C * HW) != full


def test_factorized_prior_tables_are_valid_cdfs():
    torch.manual_seed(0)
    model = FactorizedPrior(8, 12)
    eb = model.entropy_bottleneck
    with pytest.raises(CoderInputError, match="update"):
        fast_compressai.coders.factorized.FactorizedWarpDivCodec._tables(eb)
    assert model.update(force=True)
    cdf = eb._quantized_cdf.numpy()
    sizes = eb._cdf_length.numpy()
    assert cdf.dtype == np.int32 and cdf.shape[0] == 12 and sizes.max() == cdf.shape[1]
    for c in range(12):
        row = cdf[c, :sizes[c]]
        assert row[0] == 0 and row[-1] == 65536 and (np.diff(row) >= 1).all()
    assert (eb._offset.numpy() <= 0).all()
    x = torch.rand(1, 3, 64, 64)
    out = model(x)
    assert out["x_hat"].shape == x.shape
    y = model.g_a(x)
    assert y.shape == (1, 12, 4, 4)
    med = eb._extend_ndims(eb._get_medians().detach(), 2)
    sym = eb.quantize(y, "symbols", med)
    assert sym.dtype == torch.int32
    assert torch.equal(eb.dequantize(sym, med, med.dtype), torch.round(y - med) + med)
    idx = eb._build_indexes(y.size())
    assert torch.equal(idx[0, :, 0, 0], torch.arange(12, dtype=torch.int32))
