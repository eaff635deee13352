"""User-facing entry points: ``accelerate`` and ``FastModel``.

``accelerate(model, P, ..., coder="warp_div")`` follows the reference's
warp_div branch (api.py:132-448 of the reference): validate the model and
device, deep-copy the model to CUDA, attach a ``FactorizedWarpDivCodec`` and
return a ``FastModel`` whose ``compress``/``decompress`` go through it, with
an ``AccelerationReport``.

Differences, all additive:
  * the model may be CompressAI's ``FactorizedPrior`` (when installed) or
    this package's FP32 restatement ``fast_compressai.balle.FactorizedPrior``;
  * ``transforms="bf16"`` swaps g_a / g_s for this package's sm_100a
    tensor-core layers (default ``"fp32"`` keeps the model's own modules, as
    the reference does without a precision config); ``transforms="fp8"``
    does the same with e4m3 operands (per-tensor scales, as the reference's
    FP8 candidates) for every convolution that has an e4m3 kernel;
  * a saved precision map (``precision_config_path``, the reference's
    schema-4 JSON) is applied to the B200 transforms: convolutions mapped to
    "fp8" run the e4m3 tensor-core kernels where one exists, all other
    modules run with bf16 operands, and the report's
    ``precision_applications`` records each module's requested and applied
    precision.  The map is checked against the model fingerprint, coder,
    P_ch and operator inventory as the reference does; its candidate-catalog
    fingerprint and device capability describe the reference's candidates
    and search GPU and are not compared;
  * the reference's CAIEC precision search (``calibration_data``) is not part
    of this build and raises ``ConfigurationError``.
"""

from __future__ import annotations

import copy
from dataclasses import asdict, dataclass, replace
from typing import Any, Mapping

import torch
from torch import nn

from .config import AccelerationConfig, CompileConfig, ConfigurationError
from .coders.factorized import FactorizedWarpDivCodec


@dataclass(frozen=True)
class CompileReport:
    """What the wrapper exposes (subset of the reference's CompileReport)."""

    backend: str
    accelerated: bool
    available_paths: tuple[str, ...]
    missing_paths: tuple[str, ...]
    fallback_used: bool
    message: str
    contract_family: str = "generic"
    update_called: bool = False

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


@dataclass(frozen=True)
class AccelerationReport:
    """Status of ``accelerate`` (same fields as the reference, api.py:88-124)."""

    status: str
    model_class: str
    adapter_family: str
    p_ch: int | None
    quality_budget: float
    quality_metric: str
    profiling_status: str
    precision_selection_status: str
    selected_candidate: str
    psnr_drop_db: float | None
    reference_latency_ms: float | None
    candidate_latency_ms: float | None
    coder_status: str
    p_ch_applied: bool
    runtime_status: str
    speedup: float | None
    message: str
    rd_cost: float | None = None
    budget_met: bool | None = None
    precision_config_path: str | None = None
    sensitivity_probe_count: int = 0
    unavailable_probe_count: int = 0
    recovered_instance_count: int = 0
    p_ch_selection_status: str = "explicit"
    p_ch_selection_reason: str | None = None
    p_ch_sweep: tuple[Mapping[str, Any], ...] = ()
    # (module_path, requested, applied, reason) per conv / GDN module when a
    # precision map was applied (additive: not in the reference's report)
    precision_applications: tuple[tuple[str, str, str, str | None], ...] = ()

    @property
    def accelerated(self) -> bool:
        return self.runtime_status == "applied" and self.speedup is not None and self.speedup > 1.0

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


def _is_factorized_prior(model: nn.Module) -> bool:
    from .balle import FactorizedPrior as OwnFactorizedPrior

    if type(model) is OwnFactorizedPrior:
        return True
    try:
        from compressai.models import FactorizedPrior
    except ImportError:
        return False
    return type(model) is FactorizedPrior


_TRANSFORMS = ("fp32", "bf16", "fp8")


def accelerate(
    model: nn.Module,
    P: int | None = None,
    budget: float | None = None,
    *,
    config: AccelerationConfig | Mapping[str, Any] | None = None,
    device: str | None = None,
    sample: Any | None = None,
    coder: str | None = None,
    calibration_data: Any | None = None,
    dataset_name: str | None = None,
    precision_config_path: str | None = None,
    precision_config_output_dir: Any | None = None,
    transforms: str = "fp32",
) -> "FastModel":
    """Attach the B200 warp_div GA-ANS coder (and optionally B200 transforms) to a FactorizedPrior."""
    if not isinstance(model, nn.Module):
        raise TypeError(f"model must be an instance of torch.nn.Module, got {type(model).__name__}")
    cfg = AccelerationConfig.from_value(config, P=P, budget=budget, device=device, coder=coder,
                                        precision_config_path=precision_config_path)
    if precision_config_path is not None and calibration_data is not None:
        raise ConfigurationError("do not combine precision_config_path with calibration_data")
    if transforms not in _TRANSFORMS:
        raise ConfigurationError(f"transforms must be one of {_TRANSFORMS}")
    del precision_config_output_dir
    codec = None
    runtime_model = model
    target = None
    p_selection = p_sweep = None
    if cfg.coder == "warp_div":
        if not _is_factorized_prior(model):
            raise ConfigurationError("warp_div currently supports only CompressAI FactorizedPrior")
        if sample is not None:
            raise ConfigurationError("warp_div precision selection uses calibration_data; legacy sample "
                                     "profiling is unavailable")
        if not torch.cuda.is_available():
            raise ConfigurationError("warp_div requires CUDA")
        target = torch.device(cfg.device or "cuda")
        if target.type != "cuda":
            raise ConfigurationError("warp_div requires device='cuda'")
        if calibration_data is not None:
            # This build selects P_ch from calibration data (the reference's
            # sweep, api.py:255-263); the CAIEC precision search that the
            # reference runs first is not part of it.
            from .profiling import CalibrationData

            if P is not None or cfg.p_ch is not None:
                raise ConfigurationError("CAIEC precision selection is not part of this build; calibration_data "
                                         "selects P_ch when P is None")
            if not isinstance(calibration_data, CalibrationData):
                raise ConfigurationError("calibration_data must be a CalibrationData object prepared outside "
                                         "accelerate()")
            if dataset_name is not None and dataset_name != calibration_data.dataset_name:
                raise ConfigurationError("dataset_name does not match calibration_data")
        precision_config = None
        layer_precisions = None
        if cfg.precision_config_path is not None:
            precision_config, layer_precisions = _load_precision_map(cfg.precision_config_path, model, cfg)
        runtime_model = copy.deepcopy(model).to(target).eval()
        if transforms != "fp32" or precision_config is not None:
            from .transforms import convert_factorized_prior

            if precision_config is not None and transforms != "fp32":
                raise ConfigurationError("a precision config selects the transform precisions; leave "
                                         "transforms at its default")
            runtime_model = convert_factorized_prior(runtime_model,
                                                     precision="fp8" if transforms == "fp8" else "bf16",
                                                     layer_precisions=layer_precisions)
            transforms = transforms if precision_config is None else "precision_map"
        p_ch = cfg.p_ch if cfg.p_ch is not None else 1
        if precision_config is not None:
            p_ch = precision_config.p_ch
        if calibration_data is not None:
            from .profiling import sweep_p_ch

            p_selection, p_sweep = sweep_p_ch(runtime_model, calibration_data, model_name=type(model).__qualname__,
                                              warmup=1, repetitions=1)
            p_ch = p_selection.selected_p_ch
        codec = FactorizedWarpDivCodec(runtime_model, p_ch)
    elif sample is not None:
        raise ConfigurationError("the legacy BF16 sample profiling of coder='rans' is not part of this build")

    wrapped = FastModel(runtime_model, CompileConfig(device=str(target) if target is not None else cfg.device))
    applied = codec is not None and transforms != "fp32"
    if codec is not None:
        wrapped._coder = codec
        message = (
            "The B200 warp_div GA-ANS coder is applied to compress/decompress and P_ch is applied; "
            f"transforms run in {transforms}. Payloads remain device-local."
        )
    else:
        message = "Reference wrapper returned. P was recorded as GA-ANS p_ch; no precision candidate was applied."
    wrapped.acceleration_config = cfg
    wrapped.acceleration_report = AccelerationReport(
        status="coder_applied" if codec is not None else "reference_only",
        model_class=type(model).__qualname__,
        adapter_family=wrapped.report.contract_family,
        p_ch=codec.p_ch if codec is not None else cfg.p_ch,
        quality_budget=float(cfg.budget),
        quality_metric="psnr_drop_db",
        profiling_status="not_run",
        precision_selection_status="selected" if applied else "not_run",
        selected_candidate=transforms if codec is not None else "fp32",
        psnr_drop_db=None,
        reference_latency_ms=None,
        candidate_latency_ms=None,
        coder_status="warp_div" if codec is not None else "rans",
        p_ch_applied=codec is not None,
        runtime_status="applied" if applied else "not_applied",
        speedup=None,
        message=message,
        p_ch_selection_status="explicit" if P is not None or cfg.p_ch is not None else "default",
    )
    if codec is not None and precision_config is not None:
        apps = tuple(runtime_model.g_a.precision_notes) + tuple(runtime_model.g_s.precision_notes)
        wrapped.acceleration_report = replace(
            wrapped.acceleration_report,
            precision_selection_status="loaded_from_config",
            selected_candidate="precision_map",
            rd_cost=float(precision_config.validated_rd_cost),
            budget_met=bool(precision_config.budget_met),
            precision_config_path=str(cfg.precision_config_path),
            sensitivity_probe_count=len(precision_config.probe_records),
            unavailable_probe_count=sum(1 for r in precision_config.probe_records
                                        if r.get("unavailable_reason") is not None),
            recovered_instance_count=len(precision_config.recovery_order),
            p_ch_selection_status="loaded_from_config",
            p_ch_selection_reason=(precision_config.p_ch_selection or {}).get("reason"),
            p_ch_sweep=tuple((precision_config.p_ch_selection or {}).get("measurements", ())),
            precision_applications=apps,
        )
    elif codec is not None and transforms == "fp8":
        apps = tuple(runtime_model.g_a.precision_notes) + tuple(runtime_model.g_s.precision_notes)
        wrapped.acceleration_report = replace(wrapped.acceleration_report, precision_applications=apps)
    if codec is not None and p_selection is not None:
        wrapped.acceleration_report = replace(
            wrapped.acceleration_report, p_ch_selection_status=p_selection.status,
            p_ch_selection_reason=p_selection.reason, p_ch_sweep=p_sweep)
    return wrapped


def _load_precision_map(path, model: nn.Module, cfg: AccelerationConfig):
    """Load and check a saved precision config (the reference's api.py:193-236
    checks, less the candidate-catalog fingerprint and device capability):
    returns the config and its module_path -> precision map."""
    from .configs.precision import PrecisionConfig, PrecisionConfigError, model_fingerprint

    try:
        config = PrecisionConfig.load(path)
    except PrecisionConfigError as exc:
        raise ConfigurationError(str(exc)) from exc
    if config.model_fingerprint != model_fingerprint(model):
        raise ConfigurationError("precision config model fingerprint does not match the input model")
    if config.coder != cfg.coder or config.p_ch != (cfg.p_ch or 1):
        raise ConfigurationError("precision config coder/P_ch does not match the request")
    if config.device_type != "cuda":
        raise ConfigurationError("precision config was not made for a CUDA device")
    expected = {f"{t}.{i}" for t in ("g_a", "g_s") for i in range(7)}
    paths = {a.module_path for a in config.assignments}
    if paths != expected:
        raise ConfigurationError("precision config operator inventory does not match the current model")
    return config, config.precision_by_path()


class FastModel(nn.Module):
    """Wrapper that preserves a model's public compression paths (api.py:451-532 of the reference)."""

    def __init__(self, model: nn.Module, config: CompileConfig, *, report: CompileReport | None = None) -> None:
        super().__init__()
        self.model = model
        self.config = config
        available = tuple(name for name in ("forward", "compress", "decompress") if hasattr(model, name))
        missing = tuple(name for name in ("compress", "decompress") if not hasattr(model, name))
        self._report = report or CompileReport(
            backend=config.backend,
            accelerated=False,
            available_paths=available,
            missing_paths=missing,
            fallback_used=bool(missing) and config.enable_reference_fallback,
            message="Reference backend selected; no low-precision or graph optimization was applied.",
            contract_family="compressai" if hasattr(model, "entropy_bottleneck") else "generic",
        )
        if config.device is not None:
            self.to(config.device)

    @property
    def report(self) -> CompileReport:
        return self._report

    def forward(self, *args: Any, **kwargs: Any) -> Any:
        return self.model(*args, **kwargs)

    def compress(self, *args: Any, **kwargs: Any) -> Any:
        coder = self.__dict__.get("_coder")
        if coder is not None:
            return coder.compress(*args, **kwargs)
        return self.model.compress(*args, **kwargs)

    def decompress(self, *args: Any, **kwargs: Any) -> Any:
        coder = self.__dict__.get("_coder")
        if coder is not None:
            return coder.decompress(*args, **kwargs)
        return self.model.decompress(*args, **kwargs)

    def compress_async(self, x) -> Any:
        """Enqueue compress() and return a handle whose result() waits for
        the payload size alone (warp_div coder only): the overlap of
        execution_mode="overlap", see FactorizedWarpDivCodec.compress_async."""
        return self._host_coder("compress_async").compress_async(x)

    def upload_host(self, x, **kwargs: Any) -> Any:
        """Start the upload of a host batch and return a handle for compress() (warp_div coder only)."""
        return self._host_coder("upload_host").upload_host(x, **kwargs)

    def compress_host(self, x, **kwargs: Any) -> Any:
        """compress() of a host batch, its upload overlapped with g_a (warp_div coder only)."""
        return self._host_coder("compress_host").compress_host(x, **kwargs)

    def decompress_host(self, strings, shape, out=None, **kwargs: Any) -> Any:
        """decompress() into host memory, the download overlapped with g_s (warp_div coder only)."""
        return self._host_coder("decompress_host").decompress_host(strings, shape, out, **kwargs)

    def _host_coder(self, name: str):
        coder = self.__dict__.get("_coder")
        if coder is None or not hasattr(coder, name):
            raise ConfigurationError(f"{name} needs a model accelerated with coder='warp_div'")
        return coder

    def update(self, *args: Any, **kwargs: Any) -> Any:
        result = self.model.update(*args, **kwargs)
        self._report = replace(self._report, update_called=True)
        return result

    def state_dict(self, *args: Any, **kwargs: Any) -> Any:
        return self.model.state_dict(*args, **kwargs)

    def load_state_dict(self, *args: Any, **kwargs: Any) -> Any:
        return self.model.load_state_dict(*args, **kwargs)

    def __getattr__(self, name: str) -> Any:
        try:
            return super().__getattr__(name)
        except AttributeError:
            modules = object.__getattribute__(self, "_modules")
            model = modules.get("model")
            if model is not None:
                return getattr(model, name)
            raise


def compile(model: nn.Module, config: CompileConfig | Mapping[str, Any] | None = None) -> FastModel:
    """Reference-path wrapper (no operator rewriting)."""
    if not isinstance(model, nn.Module):
        raise TypeError(f"model must be an instance of torch.nn.Module, got {type(model).__name__}")
    return FastModel(model, CompileConfig.from_value(config))


def optimize(model: nn.Module, config: CompileConfig | Mapping[str, Any] | None = None) -> FastModel:
    """Alias of ``compile``."""
    return compile(model, config=config)
