"""Entropy coder backends: the B200 ``warp_div`` coder and its payload type."""

from .capabilities import CoderCapability, coder_catalog, create_coder, warp_div_capability
from .compressai_ans import CompressAIANSBackend
from .errors import BitstreamError, CoderDependencyError, CoderError, CoderInputError, CoderStateError
from .warp_div import WarpDivBackend, WarpDivPayload

__all__ = [
    "BitstreamError",
    "CoderCapability",
    "CoderDependencyError",
    "CoderError",
    "CoderInputError",
    "CoderStateError",
    "CompressAIANSBackend",
    "WarpDivBackend",
    "WarpDivPayload",
    "coder_catalog",
    "create_coder",
    "warp_div_capability",
]
