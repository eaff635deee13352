"""P_ch selection on the B200: ``sweep_p_ch`` measures every candidate on
calibration images through the accelerated model and ``accelerate(P=None,
calibration_data=...)`` attaches the coder at the chosen P_ch, recording the
sweep in its report (the reference's api.py:255-263 flow, without the CAIEC
precision search that precedes it there)."""

from __future__ import annotations

import pytest
import torch

from fast_compressai import (
    CalibrationData,
    ConfigurationError,
    accelerate,
    calibration_from_images,
    choose_p_ch,
    sweep_p_ch,
)
from tests.model_inputs import smooth_images, spread_latent_prior

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def setup(cuda_device):
    x = smooth_images(2, 256, 384, seed=31, device=cuda_device)
    model = spread_latent_prior(128, 192, x, target_std=12.0)
    return model, calibration_from_images(x, "synthetic-smooth-noise")


def test_calibration_data_contract(setup, cuda_device):
    _, cal = setup
    assert isinstance(cal, CalibrationData) and len(cal.samples) == 2
    assert all(s.shape == (1, 3, 256, 384) and s.device.type == "cuda" for s in cal.samples)
    assert torch.equal(cal.raw_targets[0], cal.samples[0] * 255.0)
    with pytest.raises(ValueError, match="lie in"):
        calibration_from_images(torch.full((1, 3, 8, 8), 2.0), "bad")


def test_sweep_measures_every_candidate_and_applies_the_rule(setup):
    model, cal = setup
    fast = accelerate(model, P=4, device="cuda:0", transforms="bf16")
    candidates = (1, 2, 4, 8, 16)
    selection, ms = sweep_p_ch(fast.model, cal, candidates=candidates, warmup=1, repetitions=2)
    assert tuple(m["p_ch"] for m in ms) == candidates
    for m in ms:
        assert m["inference_total_ms"] > 0 and m["codec_total_ms"] > 0 and m["bpp"] > 0
        assert m["codec_total_ms"] == pytest.approx(m["compress_codec_ms"] + m["decompress_codec_ms"])
        assert m["selected"] == (m["p_ch"] == selection.selected_p_ch)
    # the choice is the rule's on these measurements
    again = choose_p_ch(ms)
    assert (again.selected_p_ch, again.status) == (selection.selected_p_ch, selection.status)
    # a larger P_ch gives fewer, longer chunks, so less padding and fewer
    # initial states: the payload shrinks
    bpp = [m["bpp"] for m in ms]
    assert bpp[-1] < bpp[0]
    # the coder is lossless: the reconstruction is the same whatever the chunking
    assert max(m["psnr_db"] for m in ms) - min(m["psnr_db"] for m in ms) < 1e-6


def test_accelerate_selects_p_from_calibration_data(setup):
    model, cal = setup
    fast = accelerate(model, device="cuda:0", transforms="bf16", calibration_data=cal)
    rep = fast.acceleration_report
    assert rep.p_ch_selection_status in ("auto_selected", "fallback_closest_balance")
    assert rep.p_ch_selection_reason in ("largest_relative_error_pass", "no_candidate_within_relative_tolerance")
    chosen = [m["p_ch"] for m in rep.p_ch_sweep if m["selected"]]
    assert chosen == [rep.p_ch] and fast._coder.p_ch == rep.p_ch
    assert [m["p_ch"] for m in rep.p_ch_sweep][:4] == [1, 2, 3, 4]
    with torch.inference_mode():
        out = fast.compress(cal.samples[0])
        x_hat = fast.decompress(out["strings"], out["shape"])["x_hat"]
    assert out["strings"][0].p_ch == rep.p_ch and x_hat.shape == cal.samples[0].shape


def test_calibration_data_is_only_for_choosing_p(setup):
    model, cal = setup
    with pytest.raises(ConfigurationError, match="selects P_ch when P is None"):
        accelerate(model, P=4, device="cuda:0", calibration_data=cal)
    with pytest.raises(ConfigurationError, match="CalibrationData"):
        accelerate(model, device="cuda:0", calibration_data=[cal.samples[0]])
    with pytest.raises(ConfigurationError, match="dataset_name"):
        accelerate(model, device="cuda:0", calibration_data=cal, dataset_name="kodak")
