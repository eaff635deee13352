"""Saved per-operator precision maps (the output of the reference's CAIEC search).

Reads and writes the reference's versioned JSON (configs/precision.py:1-294
of the reference, schema 4): the same field set, validation rules, error
type and messages, and ``model_fingerprint`` (SHA-256 over the sorted
state dict: name, dtype, shape as compact JSON, raw bytes;
configs/precision.py:245-254), so a map saved by the reference for a model
loads here against the same weights.  The search that produces the map
(policies/caiec_selection.py) is not part of this build; ``accelerate``
applies a loaded map to the B200 transform layers.
"""

from __future__ import annotations

import hashlib
import json
import math
import os
import re
import tempfile
from dataclasses import asdict, dataclass, fields
from pathlib import Path
from typing import Any, Mapping

PRECISION_CONFIG_SCHEMA_VERSION = 4
RD_COST_FORMULA = "log10(bpp/bpp_ref)+(psnr_ref-psnr)"
_HEX = frozenset("0123456789abcdef")


class PrecisionConfigError(ValueError):
    """Raised when a precision config cannot safely be loaded or applied."""


def _finite(value: Any, name: str) -> None:
    if isinstance(value, bool) or not isinstance(value, (int, float)) or not math.isfinite(float(value)):
        raise PrecisionConfigError(f"{name} must be finite")


def _plain(value: Any, path: str) -> Any:
    """JSON-safe copy of value (str / bool / int / finite float / lists / string-keyed maps)."""
    if value is None or isinstance(value, (str, bool)) or type(value) is int:
        return value
    if type(value) is float:
        _finite(value, path)
        return value
    if isinstance(value, (list, tuple)):
        return [_plain(item, f"{path}[]") for item in value]
    if isinstance(value, Mapping):
        out = {}
        for key, item in value.items():
            if not isinstance(key, str):
                raise PrecisionConfigError(f"{path} keys must be strings")
            out[key] = _plain(item, f"{path}.{key}")
        return out
    raise PrecisionConfigError(f"{path} contains unsupported value {type(value).__name__}")


def _is_sha256(value: Any) -> bool:
    return isinstance(value, str) and len(value) == 64 and _HEX.issuperset(value)


@dataclass(frozen=True)
class PrecisionAssignment:
    """The precision chosen for one operator instance (a conv or GDN module)."""

    instance_id: str
    module_path: str
    logical_op: str
    candidate_key: Mapping[str, Any]
    precision: str
    backend: str
    category: str
    probe_rd_cost: float
    probe_thr_gain: float
    fallback_reason: str | None = None
    selection_reason: Any = None

    def __post_init__(self) -> None:
        for name in ("instance_id", "module_path", "logical_op", "precision", "backend", "category"):
            value = getattr(self, name)
            if not isinstance(value, str) or not value:
                raise PrecisionConfigError(f"assignment {name} must be non-empty")
        _finite(self.probe_rd_cost, "probe_rd_cost")
        _finite(self.probe_thr_gain, "probe_thr_gain")
        if not isinstance(self.candidate_key, Mapping):
            raise PrecisionConfigError("candidate_key must be a mapping")
        _plain(dict(self.candidate_key), "candidate_key")


_FIELDS = (
    "schema_version", "kind", "model_name", "model_fingerprint", "dataset_name", "dataset_fingerprint",
    "dataset_sample_count", "device_type", "device_capability", "coder", "p_ch", "epsilon", "rd_cost_formula",
    "selector_version", "catalog_fingerprint", "assignments", "probe_records", "validated_rd_cost", "budget_met",
    "recovery_order", "recovery_steps", "records_path", "recovery_path", "p_ch_selection", "profile_cost_ms",
    "created_utc",
)


@dataclass(frozen=True)
class PrecisionConfig:
    model_name: str
    model_fingerprint: str
    dataset_name: str
    dataset_fingerprint: str
    device_type: str
    device_capability: tuple[int, int]
    coder: str
    p_ch: int | None
    epsilon: float
    rd_cost_formula: str
    selector_version: str
    catalog_fingerprint: str
    assignments: tuple[PrecisionAssignment, ...]
    probe_records: tuple[Mapping[str, Any], ...]
    validated_rd_cost: float
    budget_met: bool
    created_utc: str
    dataset_sample_count: int
    profile_cost_ms: float
    recovery_order: tuple[str, ...] = ()
    recovery_steps: tuple[Mapping[str, Any], ...] = ()
    records_path: str | None = None
    recovery_path: str | None = None
    p_ch_selection: Mapping[str, Any] | None = None
    schema_version: int = PRECISION_CONFIG_SCHEMA_VERSION

    def __post_init__(self) -> None:
        if type(self.schema_version) is not int or self.schema_version != PRECISION_CONFIG_SCHEMA_VERSION:
            raise PrecisionConfigError(f"unsupported precision config schema {self.schema_version!r}")
        for name in ("model_name", "dataset_name", "device_type", "coder", "selector_version"):
            if not isinstance(getattr(self, name), str) or not getattr(self, name):
                raise PrecisionConfigError(f"{name} must be a non-empty string")
        for name in ("model_fingerprint", "dataset_fingerprint", "catalog_fingerprint"):
            if not _is_sha256(getattr(self, name)):
                raise PrecisionConfigError(f"{name} must be a SHA-256 hex digest")
        if self.rd_cost_formula != RD_COST_FORMULA:
            raise PrecisionConfigError("unsupported RD Cost formula")
        for name in ("epsilon", "validated_rd_cost", "profile_cost_ms"):
            _finite(getattr(self, name), name)
        if self.epsilon < 0 or self.profile_cost_ms < 0:
            raise PrecisionConfigError("epsilon and profile cost must be non-negative")
        if self.p_ch is not None and (type(self.p_ch) is not int or self.p_ch <= 0):
            raise PrecisionConfigError("p_ch must be a positive integer or None")
        if type(self.dataset_sample_count) is not int or self.dataset_sample_count < 1:
            raise PrecisionConfigError("dataset_sample_count must be positive")
        if len(self.device_capability) != 2 or any(type(v) is not int for v in self.device_capability):
            raise PrecisionConfigError("device_capability must be an integer pair")
        for name in ("probe_records", "recovery_steps"):
            for record in getattr(self, name):
                if not isinstance(record, Mapping):
                    raise PrecisionConfigError(f"{name} must contain mappings")
                _plain(dict(record), name)
        for name in ("records_path", "recovery_path"):
            value = getattr(self, name)
            if value is not None and (not isinstance(value, str) or not value):
                raise PrecisionConfigError(f"{name} must be a non-empty string or None")
        if self.p_ch_selection is not None:
            _plain(dict(self.p_ch_selection), "p_ch_selection")
        paths = [a.module_path for a in self.assignments]
        if len(paths) != len(set(paths)):
            raise PrecisionConfigError("precision assignments contain duplicate module paths")
        if any(not isinstance(a, PrecisionAssignment) for a in self.assignments):
            raise PrecisionConfigError("assignments must contain PrecisionAssignment values")

    # -- serialisation ------------------------------------------------------
    def to_dict(self) -> dict[str, Any]:
        out: dict[str, Any] = {"schema_version": self.schema_version, "kind": "fast_compressai_precision_config"}
        for f in fields(self):
            if f.name == "schema_version":
                continue
            value = getattr(self, f.name)
            if f.name == "assignments":
                value = [asdict(a) for a in value]
            elif f.name in ("probe_records", "recovery_steps"):
                value = [_plain(dict(r), f.name) for r in value]
            elif f.name in ("device_capability", "recovery_order"):
                value = list(value)
            elif f.name == "p_ch_selection" and value is not None:
                value = _plain(dict(value), f.name)
            out[f.name] = value
        return out

    @classmethod
    def from_dict(cls, value: Mapping[str, Any]) -> "PrecisionConfig":
        if not isinstance(value, Mapping) or set(value) != set(_FIELDS):
            raise PrecisionConfigError("precision config has missing or unknown fields")
        if value["kind"] != "fast_compressai_precision_config":
            raise PrecisionConfigError("invalid precision config kind")
        try:
            kwargs = {k: value[k] for k in _FIELDS if k != "kind"}
            kwargs["device_capability"] = tuple(value["device_capability"])
            kwargs["assignments"] = tuple(PrecisionAssignment(**item) for item in value["assignments"])
            kwargs["probe_records"] = tuple(value["probe_records"])
            kwargs["recovery_order"] = tuple(value["recovery_order"])
            kwargs["recovery_steps"] = tuple(value["recovery_steps"])
            return cls(**kwargs)
        except PrecisionConfigError:
            raise
        except (TypeError, ValueError, KeyError) as exc:
            raise PrecisionConfigError(f"invalid precision config: {exc}") from exc

    def to_json(self) -> str:
        return json.dumps(self.to_dict(), sort_keys=True, indent=2, ensure_ascii=False, allow_nan=False)

    @classmethod
    def from_json(cls, value: str) -> "PrecisionConfig":
        try:
            data = json.loads(value)
        except (TypeError, json.JSONDecodeError) as exc:
            raise PrecisionConfigError("precision config is not valid JSON") from exc
        return cls.from_dict(data)

    def save(self, path: str | Path) -> Path:
        """Atomic write (temporary file in the target directory, then rename)."""
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        fd, tmp = tempfile.mkstemp(prefix=f".{path.name}.", suffix=".tmp", dir=path.parent)
        try:
            with os.fdopen(fd, "w", encoding="utf-8") as handle:
                handle.write(self.to_json())
                handle.flush()
                os.fsync(handle.fileno())
            os.replace(tmp, path)
        except Exception:
            try:
                os.unlink(tmp)
            except OSError:
                pass
            raise
        return path

    @classmethod
    def load(cls, path: str | Path) -> "PrecisionConfig":
        path = Path(path)
        try:
            return cls.from_json(path.read_text(encoding="utf-8"))
        except OSError as exc:
            raise PrecisionConfigError(f"cannot read precision config {path}: {exc}") from exc

    def validate_compatibility(self, **actual: Any) -> None:
        names = ("model_fingerprint", "dataset_fingerprint", "device_type", "device_capability", "coder", "p_ch",
                 "catalog_fingerprint")
        bad = [n for n in names if n in actual and getattr(self, n) != actual[n]]
        if bad:
            raise PrecisionConfigError("precision config is incompatible: " + ", ".join(bad))

    def precision_by_path(self) -> dict[str, str]:
        """module_path -> precision ("fp8", "fp16", "bf16" or "fp32")."""
        return {a.module_path: a.precision for a in self.assignments}


def model_fingerprint(model: Any) -> str:
    """SHA-256 over the model's state dict in name order: for each tensor its
    name, dtype string, shape as compact JSON and contiguous CPU bytes."""
    digest = hashlib.sha256()
    for name, tensor in sorted(model.state_dict().items()):
        value = tensor.detach().contiguous().cpu()
        digest.update(name.encode("utf-8"))
        digest.update(str(value.dtype).encode("ascii"))
        digest.update(json.dumps(list(value.shape), separators=(",", ":")).encode("ascii"))
        digest.update(value.numpy().tobytes())
    return digest.hexdigest()


def fingerprint_json(value: Any) -> str:
    data = json.dumps(value, sort_keys=True, separators=(",", ":"), allow_nan=False).encode("utf-8")
    return hashlib.sha256(data).hexdigest()


def _safe_name(value: str) -> str:
    value = re.sub(r"[^A-Za-z0-9_.-]+", "_", value.strip()).strip("._-")
    if not value or value in {".", ".."}:
        raise PrecisionConfigError("model/dataset name is not a safe path component")
    return value[:120]
