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
from .policies import PChSelection, choose_p_ch, legal_p_candidates
from .profiling import CalibrationData, calibration_from_images, default_p_candidates, sweep_p_ch

__all__ = [
    "AccelerationConfig",
    "AccelerationReport",
    "BitstreamError",
    "CalibrationData",
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
    "PChSelection",
    "UnsupportedOperationError",
    "WarpDivBackend",
    "WarpDivPayload",
    "accelerate",
    "calibration_from_images",
    "choose_p_ch",
    "coder_catalog",
    "compile",
    "create_coder",
    "default_p_candidates",
    "legal_p_candidates",
    "optimize",
    "sweep_p_ch",
    "warp_div_capability",
]

__version__ = "0.1.0"
