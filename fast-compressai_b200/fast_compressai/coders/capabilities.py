"""Coder capability discovery without loading the native library.

Mirrors coders/capabilities.py:20-49 of the reference: availability is
decided by ``importlib.util.find_spec("fast_compressai.coders._warp_div")``
plus, here, the presence of the built C-ABI library that module binds.
"""

from __future__ import annotations

import importlib.util
from dataclasses import dataclass

import torch

from .. import _native


@dataclass(frozen=True)
class CoderCapability:
    backend: str
    available: bool
    reason: str | None
    device: str | None
    persistent_payload: bool


def warp_div_capability(device: torch.device | str | None = None) -> CoderCapability:
    requested = torch.device(device) if device is not None else None
    if not torch.cuda.is_available():
        return CoderCapability("warp_div", False, "CUDA runtime/device unavailable", None, False)
    if requested is not None and requested.type != "cuda":
        return CoderCapability("warp_div", False, "warp_div requires a CUDA device", str(requested), False)
    where = str(requested or torch.device("cuda"))
    spec = importlib.util.find_spec("fast_compressai.coders._warp_div")
    if spec is None or not _native.available():
        return CoderCapability("warp_div", False, "optional CUDA extension is not built", where, False)
    major, _minor = torch.cuda.get_device_capability(requested)
    if major != 10:
        return CoderCapability("warp_div", False, "this build targets sm_100a (B200) devices only", where, False)
    return CoderCapability("warp_div", True, None, where, False)


def coder_catalog() -> tuple[str, ...]:
    """Return exactly the supported entropy coder backend identifiers."""

    return ("compressai-rans", "warp_div")


def create_coder(name: str):
    """Construct one supported backend without loading unrelated backends."""

    if name == "compressai-rans":
        from .compressai_ans import CompressAIANSBackend

        return CompressAIANSBackend()
    if name == "warp_div":
        from .warp_div import WarpDivBackend

        return WarpDivBackend()
    raise ValueError(f"unsupported coder {name!r}; supported coders are {coder_catalog()}")
