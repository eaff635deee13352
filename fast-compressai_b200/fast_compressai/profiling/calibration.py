"""Calibration images for measurements on the accelerated model.

``CalibrationData`` has the reference's fields and checks
(profiling/rd.py:31-53): one-image NCHW samples in [0, 1] on the CUDA
device, their raw targets in [0, 255], the dataset's name and fingerprint,
and the divide-by-255 normalisation contract.  The reference loads Kodak
from a float32 file (``load_kodak_f32``); that file is not part of this
build, so ``calibration_from_images`` wraps any batch of images in [0, 1]
(for instance seeded synthetic ones) the same way.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass
from typing import Sequence

import torch


def calibration_fingerprint(samples: Sequence[torch.Tensor], dataset_name: str) -> str:
    """SHA-256 over the dataset name and each sample's dtype, shape and bytes
    (profiling/rd.py:18-26 of the reference)."""
    digest = hashlib.sha256(dataset_name.encode("utf-8"))
    for sample in samples:
        value = sample.detach().contiguous().cpu()
        digest.update(str(value.dtype).encode("ascii"))
        digest.update(repr(tuple(value.shape)).encode("ascii"))
        digest.update(value.numpy().tobytes())
    return digest.hexdigest()


@dataclass(frozen=True)
class CalibrationData:
    samples: tuple[torch.Tensor, ...]
    raw_targets: tuple[torch.Tensor, ...]
    dataset_name: str
    dataset_fingerprint: str
    normalization: str
    denormalization: str
    data_range: float

    def __post_init__(self) -> None:
        if not self.samples or len(self.samples) != len(self.raw_targets):
            raise ValueError("calibration samples and raw targets must be non-empty and paired")
        if not self.dataset_name or not self.dataset_fingerprint:
            raise ValueError("calibration dataset identity is required")
        if self.normalization != "divide_by_255" or self.denormalization != "multiply_by_255":
            raise ValueError("unsupported calibration normalization contract")
        if self.data_range != 255.0:
            raise ValueError("calibration PSNR data_range must be 255")
        for sample, target in zip(self.samples, self.raw_targets):
            if sample.shape != target.shape or sample.ndim != 4:
                raise ValueError("calibration samples and targets must share NCHW shape")
            if sample.device.type != "cuda" or target.device.type != "cuda":
                raise ValueError("calibration tensors must already be on CUDA")


def calibration_from_images(images: torch.Tensor, dataset_name: str, device="cuda") -> CalibrationData:
    """``CalibrationData`` for a batch of images [B, 3, H, W] in [0, 1]: one
    sample per image on ``device``, raw targets = 255 * sample."""
    if not isinstance(images, torch.Tensor) or images.ndim != 4:
        raise ValueError("images must be an NCHW tensor")
    if float(images.min()) < 0.0 or float(images.max()) > 1.0:
        raise ValueError("images must lie in [0, 1]")
    samples = tuple(images[i:i + 1].to(device=device, dtype=torch.float32).contiguous() for i in range(images.shape[0]))
    raw = tuple((s * 255.0).contiguous() for s in samples)
    return CalibrationData(samples=samples, raw_targets=raw, dataset_name=dataset_name,
                           dataset_fingerprint=calibration_fingerprint(samples, dataset_name),
                           normalization="divide_by_255", denormalization="multiply_by_255", data_range=255.0)
