"""Persistent configuration (saved precision maps)."""

from .precision import (PRECISION_CONFIG_SCHEMA_VERSION, PrecisionAssignment, PrecisionConfig, PrecisionConfigError,
                        model_fingerprint)

__all__ = ["PRECISION_CONFIG_SCHEMA_VERSION", "PrecisionAssignment", "PrecisionConfig", "PrecisionConfigError",
           "model_fingerprint"]
