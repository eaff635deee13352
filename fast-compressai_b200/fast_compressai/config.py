"""Public configuration objects.

``AccelerationConfig`` keeps the reference's fields, validation and override
rules (config.py:14-101 of the reference); ``CompileConfig`` keeps the
fields ``accelerate`` passes through (config.py:104-167).
"""

from __future__ import annotations

import math
from dataclasses import asdict, dataclass
from typing import Any, Mapping


class ConfigurationError(ValueError):
    """Raised when a configuration is invalid."""


_CODERS = ("warp_div", "rans")
_MODES = ("sequential", "overlap")


@dataclass(frozen=True)
class AccelerationConfig:
    """Constraints of ``accelerate``.

    ``P`` is stored as ``p_ch``: latent channels per independently coded
    GA-ANS chunk.  ``budget`` is an RD/quality budget, independent of any
    coding-time constraint."""

    p_ch: int | None = None
    budget: float = 0.0
    coder: str = "warp_div"
    device: str | None = None
    profile_path: str | None = None
    precision_config_path: str | None = None
    execution_mode: str = "sequential"

    def __post_init__(self) -> None:
        if self.p_ch is not None and (type(self.p_ch) is not int or self.p_ch <= 0):
            raise ConfigurationError("P (p_ch) must be a positive integer or None")
        if self.coder not in _CODERS:
            raise ConfigurationError("coder must be 'warp_div' or 'rans'")
        if isinstance(self.budget, bool) or not isinstance(self.budget, (int, float)):
            raise ConfigurationError("budget must be a non-negative finite RD/quality value")
        if self.budget < 0 or not math.isfinite(float(self.budget)):
            raise ConfigurationError("budget must be a non-negative finite RD/quality value")
        for name in ("device", "profile_path", "precision_config_path"):
            value = getattr(self, name)
            if value is not None and not isinstance(value, str):
                raise ConfigurationError(f"{name} must be a string or None")
        if self.execution_mode not in _MODES:
            raise ConfigurationError("execution_mode must be 'sequential' or 'overlap'")

    @classmethod
    def from_value(cls, value: "AccelerationConfig | Mapping[str, Any] | None", *, P: int | None = None,
                   budget: float | None = None, device: str | None = None, coder: str | None = None,
                   precision_config_path: str | None = None) -> "AccelerationConfig":
        overrides = {"p_ch": P, "budget": budget, "device": device, "coder": coder,
                     "precision_config_path": precision_config_path}
        if value is None:
            return cls(p_ch=P, budget=0.0 if budget is None else budget, device=device,
                       coder="warp_div" if coder is None else coder,
                       precision_config_path=precision_config_path)
        if isinstance(value, cls):
            if any(v is not None for v in overrides.values()):
                raise ConfigurationError("do not combine config with P/budget/device/coder overrides")
            return value
        if isinstance(value, Mapping):
            data = dict(value)
            if "P" in data:
                if "p_ch" in data:
                    raise ConfigurationError("use only one of P and p_ch")
                data["p_ch"] = data.pop("P")
            for key, override in overrides.items():
                if override is not None:
                    if key in data:
                        raise ConfigurationError(f"{key} specified both in config and as an argument")
                    data[key] = override
            known = {"p_ch", "budget", "coder", "device", "profile_path", "precision_config_path", "execution_mode"}
            unknown = set(data) - known
            if unknown:
                raise ConfigurationError(f"unknown acceleration config field(s): {', '.join(sorted(map(str, unknown)))}")
            try:
                return cls(**data)
            except TypeError as exc:
                raise ConfigurationError(str(exc)) from exc
        raise ConfigurationError("config must be None, AccelerationConfig, or a mapping")

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


@dataclass(frozen=True)
class CompileConfig:
    """Device placement of the wrapped model (reference-only compile path)."""

    device: str | None = None
    backend: str = "reference"
    enable_reference_fallback: bool = True
    enable_operator_fallback: bool = True
    default_precision: str = "fp32"

    def __post_init__(self) -> None:
        if self.device is not None and not isinstance(self.device, str):
            object.__setattr__(self, "device", str(self.device))
        if self.backend != "reference":
            raise ConfigurationError(f"unsupported backend {self.backend!r}; the MVP only supports 'reference'")
        if not isinstance(self.enable_reference_fallback, bool) or not isinstance(self.enable_operator_fallback, bool):
            raise ConfigurationError("fallback switches must be bools")
        if self.default_precision != "fp32":
            raise ConfigurationError(f"unsupported default precision {self.default_precision!r}; "
                                     "the default must remain 'fp32'")

    @classmethod
    def from_value(cls, value: "CompileConfig | Mapping[str, Any] | None") -> "CompileConfig":
        if value is None:
            return cls()
        if isinstance(value, cls):
            return value
        if isinstance(value, Mapping):
            known = {"device", "backend", "enable_reference_fallback", "enable_operator_fallback", "default_precision"}
            unknown = set(value) - known
            if unknown:
                raise ConfigurationError(f"unknown compile configuration field(s): {', '.join(sorted(map(str, unknown)))}")
            try:
                return cls(**dict(value))
            except TypeError as exc:
                raise ConfigurationError(str(exc)) from exc
        raise ConfigurationError("config must be None, CompileConfig, or a mapping of configuration fields")

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)
