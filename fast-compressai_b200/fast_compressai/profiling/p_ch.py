"""P_ch sweep on the accelerated model (the reference's profiling/p_ch.py:
16-84 and the per-candidate measurement of profiling/rd.py:104-240).

For each candidate, every calibration image is compressed and decompressed
through ``FactorizedWarpDivCodec`` with its timing split (CUDA events around
the analysis transform, the encode, the decode and the synthesis transform),
after ``warmup`` untimed passes; medians over images and repetitions give
the inference time (analysis + synthesis) and the codec time (encode +
decode) that ``choose_p_ch`` balances.  bpp is payload bits per input value
(header included), PSNR is against the image.  On this build the transforms
are whatever ``accelerate`` attached (bf16 / fp8 tensor-core kernels or the
FP32 torch modules) and the coder is the B200 warp_div coder, so the choice
reflects B200 timings.
"""

from __future__ import annotations

import math
import statistics
import time
from typing import Sequence

import torch

from ..coders.factorized import FactorizedWarpDivCodec
from ..policies.p_ch import choose_p_ch, legal_p_candidates
from .calibration import CalibrationData

_DEFAULT_CANDIDATES = (1, 2, 3, 4, 6, 8, 12, 16, 24, 32, 48, 64, 96, 128, 192, 256)


def default_p_candidates(channel_count: int) -> tuple[int, ...]:
    return legal_p_candidates(channel_count, _DEFAULT_CANDIDATES)


def measure_p_ch(model, calibration: CalibrationData, p_ch: int, *, warmup: int = 1, repetitions: int = 3) -> dict:
    """One candidate's timings, bpp and PSNR on the calibration images."""
    if warmup < 0 or repetitions < 1:
        raise ValueError("warmup must be non-negative and repetitions positive")
    device = calibration.samples[0].device
    codec = FactorizedWarpDivCodec(model, p_ch)
    keys = ("compress_inference_ms", "compress_codec_ms", "decompress_codec_ms", "decompress_inference_ms")
    times = {k: [] for k in keys}
    compress_ms, decompress_ms = [], []
    bits = values = 0
    squared_error = 0.0
    with torch.inference_mode():
        for sample, raw in zip(calibration.samples, calibration.raw_targets):
            if sample.shape[0] != 1:
                raise ValueError("calibration samples must contain one image each")
            for _ in range(warmup):
                out = codec.compress(sample)
                codec.decompress(out["strings"], out["shape"])
            for _ in range(repetitions):
                timing: dict[str, float] = {}
                torch.cuda.synchronize(device)
                t0 = time.perf_counter()
                out = codec.compress(sample, timing=timing)
                torch.cuda.synchronize(device)
                t1 = time.perf_counter()
                x_hat = codec.decompress(out["strings"], out["shape"], timing=timing)["x_hat"]
                torch.cuda.synchronize(device)
                t2 = time.perf_counter()
                compress_ms.append((t1 - t0) * 1e3)
                decompress_ms.append((t2 - t1) * 1e3)
                for k in keys:
                    times[k].append(timing[k])
                bits += out["strings"][0].packed.numel() * 8
                values += sample.numel()
                squared_error += float((x_hat.float() * 255.0 - raw.float()).square().sum())
    med = {k: statistics.median(v) for k, v in times.items()}
    mse = squared_error / values
    psnr = 0.0 if mse == 0 else 20.0 * math.log10(255.0) - 10.0 * math.log10(mse)
    inference = med["compress_inference_ms"] + med["decompress_inference_ms"]
    codec_total = med["compress_codec_ms"] + med["decompress_codec_ms"]
    return {
        "p_ch": p_ch,
        "bpp": bits / values,
        "psnr_db": psnr if math.isfinite(psnr) else 0.0,
        "compress_latency_ms": statistics.median(compress_ms),
        "decompress_latency_ms": statistics.median(decompress_ms),
        **med,
        "inference_total_ms": inference,
        "codec_total_ms": codec_total,
        "codec_to_inference_ratio": codec_total / max(inference, 1e-12),
        "sample_count": len(calibration.samples),
        "warmup": warmup,
        "repetitions_per_sample": repetitions,
        "payload_semantics": "device_local_warp_div_packed_payload",
    }


def sweep_p_ch(model, calibration: CalibrationData, *, model_name: str = "FactorizedPrior",
               candidates: Sequence[int] | None = None, warmup: int = 1, repetitions: int = 3,
               relative_tolerance: float = 0.10, plateau_delta: float = 0.05, plateau_patience: int = 2):
    """Measure every legal candidate and choose P_ch; returns the selection and
    the measurements (each marked with its balance error and whether it
    passed and was selected)."""
    del model_name  # kept for the reference's signature
    channels = int(model.entropy_bottleneck.channels)
    p_values = legal_p_candidates(channels, candidates or default_p_candidates(channels))
    measurements = [measure_p_ch(model, calibration, p, warmup=warmup, repetitions=repetitions) for p in p_values]
    selection = choose_p_ch(measurements, relative_tolerance=relative_tolerance, plateau_delta=plateau_delta,
                            plateau_patience=plateau_patience)
    for item in measurements:
        item["relative_time_error"] = abs(item["codec_to_inference_ratio"] - 1.0)
        item["passed_balance"] = item["relative_time_error"] <= relative_tolerance
        item["selected"] = item["p_ch"] == selection.selected_p_ch
    return selection, tuple(measurements)
