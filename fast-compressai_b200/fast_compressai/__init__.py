"""fast_compressai (B200 build): the FactorizedPrior compress/decompress hot
path of fast-compressai with sm_100a kernels behind the reference's API."""

from .api import AccelerationReport, CompileReport, FastModel, accelerate, compile, optimize
from .coders import (
    BitstreamError,
    CoderCapability,
    CoderDependencyError,
    CoderError,
    CoderInputError,
    CoderStateError,
    CompressAIANSBackend,
    WarpDivBackend,
    WarpDivPayload,
    coder_catalog,
    create_coder,
    warp_div_capability,
)
from .config import AccelerationConfig, CompileConfig, ConfigurationError
from .errors import UnsupportedOperationError

__all__ = [
    "AccelerationConfig",
    "AccelerationReport",
    "BitstreamError",
    "CoderCapability",
    "CoderDependencyError",
    "CoderError",
    "CoderInputError",
    "CoderStateError",
    "CompileConfig",
    "CompileReport",
    "CompressAIANSBackend",
    "ConfigurationError",
    "FastModel",
    "UnsupportedOperationError",
    "WarpDivBackend",
    "WarpDivPayload",
    "accelerate",
    "coder_catalog",
    "compile",
    "create_coder",
    "optimize",
    "warp_div_capability",
]

__version__ = "0.1.0"
