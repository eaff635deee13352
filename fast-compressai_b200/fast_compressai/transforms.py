"""B200 tensor-core analysis / synthesis transforms of a FactorizedPrior.

``convert_factorized_prior(model, precision="bf16")`` replaces ``model.g_a``
and ``model.g_s`` by modules that run each (conv, GDN) or (deconv, IGDN) pair
as one fused sm_100a kernel (include/fcai_transforms.h):

    g_a: x fp32 NCHW -> [conv+GDN] x3 -> conv -> y fp32 NCHW
    g_s: y_hat fp32 NCHW -> NHWC bf16 -> [deconv+IGDN] x3 -> deconv -> x_hat fp32 NCHW

Activations between layers are bf16 NHWC.  This is the B200 counterpart of
the reference's BF16 candidates (backends/pytorch/bf16_operators.py:13-60),
which cast each module's input and weights to bf16 and call cuDNN; here the
GDN is fused into the producing convolution's epilogue and the first layer
reads the fp32 NCHW image directly.

Supported shapes: N = 128 latent-transform channels (the GDN tile width of
the kernels) and any M that is a multiple of 64 up to 256 (e.g. the
quality 1-5 FactorizedPrior, N=128, M=192).  Other shapes raise
``ConfigurationError``.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

from typing import Mapping

import torch
from torch import nn

from . import _native
from .config import ConfigurationError

FCAI_LAYER_CONV5S2 = 0
FCAI_LAYER_DECONV5S2 = 1
FCAI_EPI_NONE, FCAI_EPI_GDN, FCAI_EPI_IGDN = 0, 1, 2
FCAI_FMT_NHWC_BF16, FCAI_FMT_NCHW_F32 = 0, 1
FCAI_ALGO_IMPLICIT_GEMM, FCAI_ALGO_SCATTER, FCAI_ALGO_IMPLICIT_GEMM_PAIR = 0, 1, 2
FCAI_PREC_BF16, FCAI_PREC_FP8_E4M3 = 0, 1
# e4m3 (float8_e4m3fn) range and the reference's per-tensor scale floor
# (backends/pytorch/fp8_operators.py:16-17, 44-46)
FP8_MAX = 448.0
FP8_SCALE_MIN = float(torch.finfo(torch.float32).tiny)


class FcaiLayer(ctypes.Structure):
    _fields_ = [
        ("kind", ctypes.c_int32),
        ("cin", ctypes.c_int32),
        ("cout", ctypes.c_int32),
        ("npad", ctypes.c_int32),
        ("epilogue", ctypes.c_int32),
        ("in_format", ctypes.c_int32),
        ("out_format", ctypes.c_int32),
        ("clamp01", ctypes.c_int32),
        ("algorithm", ctypes.c_int32),
        ("precision", ctypes.c_int32),
        ("weight", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("gdn_beta", ctypes.c_void_p),
        ("gdn_gamma", ctypes.c_void_p),
        ("act_scale", ctypes.c_void_p),
        ("weight_scale", ctypes.c_float),
        ("out_channel_offset", ctypes.c_int32),
        ("amax_out", ctypes.c_void_p),
        ("out_channels_total", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


def _round16(v: int) -> int:
    return (v + 15) // 16 * 16


def pack_tma_weight(weight: torch.Tensor, transposed: bool, npad: int) -> torch.Tensor:
    """[25][npad][cin] bf16: entry [ky*5+kx][n][c] (conv: W[n,c,ky,kx]; deconv: W[c,n,ky,kx])."""
    w = weight.detach().float()
    if transposed:  # ConvTranspose2d weight [cin, cout, 5, 5]
        cin, cout = w.shape[0], w.shape[1]
        packed = w.permute(2, 3, 1, 0).reshape(25, cout, cin)
    else:  # Conv2d weight [cout, cin, 5, 5]
        cout, cin = w.shape[0], w.shape[1]
        packed = w.permute(2, 3, 0, 1).reshape(25, cout, cin)
    if npad > cout:
        packed = torch.cat([packed, packed.new_zeros(25, npad - cout, cin)], dim=1)
    return packed.to(torch.bfloat16).contiguous()


def fp8_weight_scale(weight: torch.Tensor) -> float:
    """Per-tensor symmetric scale of a weight as the reference computes it on
    CUDA (backends/pytorch/fp8_operators.py:44-46): amax / 448 with the Python
    float 448, which PyTorch evaluates as amax * fl32(1 / 448), floored at
    FLT_MIN; written out so that it is the same on any device."""
    amax = weight.detach().float().abs().amax().cpu()
    inv = torch.tensor(1.0 / FP8_MAX, dtype=torch.float32)
    return float(torch.clamp(amax * inv, min=FP8_SCALE_MIN))


def pack_tma_weight_fp8(weight: torch.Tensor, transposed: bool, npad: int,
                        scale: float | None = None) -> tuple[torch.Tensor, float]:
    """[25][npad][cin] e4m3 (as uint8) and its per-tensor scale: the bf16
    packing's layout with q = e4m3(clamp(w / scale, +-448)).  ``scale``
    defaults to the weight's own (a slice of a wider layer passes the whole
    layer's)."""
    w = weight.detach().float()
    if scale is None:
        scale = fp8_weight_scale(w)
    if transposed:
        cin, cout = w.shape[0], w.shape[1]
        packed = w.permute(2, 3, 1, 0).reshape(25, cout, cin)
    else:
        cout, cin = w.shape[0], w.shape[1]
        packed = w.permute(2, 3, 0, 1).reshape(25, cout, cin)
    if npad > cout:
        packed = torch.cat([packed, packed.new_zeros(25, npad - cout, cin)], dim=1)
    q = torch.clamp(packed / torch.tensor(scale, dtype=torch.float32, device=packed.device), -FP8_MAX, FP8_MAX)
    return q.to(torch.float8_e4m3fn).view(torch.uint8).contiguous(), scale


def pack_gather_weight(weight: torch.Tensor, npad: int) -> torch.Tensor:
    """Operand image of the cin=3 first layer: element (n, k) at
    (n % 8) * 8 + (n // 8) * 640 + (k // 8) * 64 + k % 8, k = c*25 + ky*5 + kx."""
    w = weight.detach().float()
    cout = w.shape[0]
    flat = torch.zeros(npad, 80, dtype=torch.float32, device=w.device)
    flat[:cout, :75] = w.reshape(cout, 75)
    n = torch.arange(npad, device=w.device).reshape(-1, 1)
    k = torch.arange(80, device=w.device).reshape(1, -1)
    pos = (n % 8) * 8 + (n // 8) * 640 + (k // 8) * 64 + k % 8
    image = torch.zeros(npad * 80, dtype=torch.float32, device=w.device)
    image[pos.reshape(-1)] = flat.reshape(-1)
    return image.to(torch.bfloat16).contiguous()


def pack_scatter_weight(weight: torch.Tensor, npad: int) -> torch.Tensor:
    """[npad][cin] bf16 for a transposed conv with few outputs: row
    (ky*5 + kx)*cout + co holds W[:, co, ky, kx]."""
    w = weight.detach().float()  # [cin, cout, 5, 5]
    cin, cout = w.shape[0], w.shape[1]
    rows = w.permute(2, 3, 1, 0).reshape(25 * cout, cin)
    if npad > rows.shape[0]:
        rows = torch.cat([rows, rows.new_zeros(npad - rows.shape[0], cin)], dim=0)
    return rows.to(torch.bfloat16).contiguous()


@dataclass
class _Layer:
    desc: FcaiLayer
    keep: tuple  # tensors the descriptor points into
    kind: int
    cout: int
    npad: int
    out_format: int
    name: str = ""
    precision: str = "bf16"
    # a layer wider than one MMA (cout > 256, fp32 NCHW output) runs as parts
    # that read the same input and write disjoint channel ranges
    parts: tuple = ()
    ref: object = None  # ctypes reference to desc, made once

    def __post_init__(self) -> None:
        if self.desc is not None:
            self.ref = ctypes.byref(self.desc)

    def flops(self, batch: int, h_in: int, w_in: int) -> float:
        """Algorithmic FLOPs: 2 * cin * 25 * cout per output (conv) or input
        (deconv) pixel, plus 2 * cout^2 per output pixel for GDN."""
        if self.parts:
            return sum(part.flops(batch, h_in, w_in) for part in self.parts)
        d = self.desc
        if self.kind == FCAI_LAYER_DECONV5S2:
            pix_in, pix_out = h_in * w_in, 4 * h_in * w_in
            f = 2.0 * batch * pix_in * d.cin * d.cout * 25  # the same for the scatter algorithm
        else:
            pix_out = ((h_in - 1) // 2 + 1) * ((w_in - 1) // 2 + 1)
            f = 2.0 * batch * pix_out * d.cin * d.cout * 25
        if d.epilogue != FCAI_EPI_NONE:
            f += 2.0 * batch * pix_out * d.cout * d.cout
        return f


# When set to a list, every layer launch appends (name, flops, start, end)
# CUDA events recorded on the launching stream (used by bench.py).
LAYER_TIMING: list | None = None


def _gdn_params(gdn: nn.Module):
    if hasattr(gdn, "effective_params"):
        beta, gamma = gdn.effective_params()
    else:  # CompressAI-style GDN: beta/gamma behind reparametrisers
        beta = gdn.beta_reparam(gdn.beta)
        gamma = gdn.gamma_reparam(gdn.gamma)
    c = beta.numel()
    return beta.detach().float().contiguous(), gamma.detach().float().reshape(c, c)


def fp8_supported(conv: nn.Module, gdn: nn.Module | None, *, first: bool, out_f32: bool) -> str | None:
    """None if the B200 FP8 kernels take this layer, else the reason they do
    not (the layer then runs with bf16 operands)."""
    if first:
        return "the first analysis layer (cin = 3) has no FP8 kernel"
    if conv.in_channels % 64:
        return "FP8 layers need a multiple of 64 input channels"
    npad = _round16(conv.out_channels)
    transposed = isinstance(conv, nn.ConvTranspose2d)
    if transposed and out_f32 and gdn is None and conv.out_channels <= 10:
        return "the scatter algorithm of the last synthesis layer has no FP8 kernel"
    if not out_f32 and (npad == 128 or (gdn is not None and npad == 192)):
        return None
    # latents: 192 channels, or 320 as two launches of 160
    if out_f32 and gdn is None and (npad in (160, 192) or (not transposed and conv.out_channels == 320)):
        return None
    return f"no FP8 kernel for {conv.out_channels} output channels with this epilogue"


def _make_layer(conv: nn.Module, gdn: nn.Module | None, *, first: bool, out_f32: bool, clamp: bool,
                pair: bool = False, precision: str = "bf16", fp8_scale: float | None = None) -> _Layer:
    transposed = isinstance(conv, nn.ConvTranspose2d)
    if (not transposed and not first and gdn is None and out_f32 and not pair
            and conv.out_channels > 256 and conv.bias is not None):
        return _make_split_layer(conv, clamp=clamp, precision=precision)
    if tuple(conv.kernel_size) != (5, 5) or tuple(conv.stride) != (2, 2) or tuple(conv.padding) != (2, 2):
        raise ConfigurationError("B200 transforms support 5x5 stride-2 padding-2 layers only")
    if transposed and tuple(conv.output_padding) != (1, 1):
        raise ConfigurationError("B200 transposed convolutions need output_padding=1")
    if conv.groups != 1 or tuple(conv.dilation) != (1, 1) or conv.bias is None:
        raise ConfigurationError("B200 transforms need groups=1, dilation=1 and a bias")
    cin = conv.in_channels
    cout = conv.out_channels
    npad = _round16(cout)
    scatter = transposed and out_f32 and gdn is None and cout <= 10
    if scatter:
        npad = _round16(25 * cout)
    if gdn is not None and npad not in (128, 192):
        raise ConfigurationError("B200 GDN fusion is built for 128- and 192-channel layers")
    if first:
        if cin != 3 or transposed:
            raise ConfigurationError("the first analysis layer must be a 3-channel convolution")
        weight = pack_gather_weight(conv.weight, npad)
    else:
        if cin % 64:
            raise ConfigurationError("B200 transforms need input channels divisible by 64")
        weight = pack_scatter_weight(conv.weight, npad) if scatter else pack_tma_weight(conv.weight, transposed, npad)
    if precision not in ("bf16", "fp8"):
        raise ConfigurationError(f"unknown B200 layer precision {precision!r}")
    w_scale = 1.0
    if precision == "fp8":
        reason = fp8_supported(conv, gdn, first=first, out_f32=out_f32)
        if reason is not None or pair:
            raise ConfigurationError(reason or "FP8 layers do not use CTA pairs")
        weight, w_scale = pack_tma_weight_fp8(conv.weight, transposed, npad, fp8_scale)
    if npad > 256:
        raise ConfigurationError("B200 transforms support up to 256 output channels per layer")
    bias = conv.bias.detach().float().contiguous()
    keep = [weight, bias]
    beta_ptr = gamma_ptr = None
    epi = FCAI_EPI_NONE
    if gdn is not None:
        beta, gamma = _gdn_params(gdn)
        gamma = gamma.to(torch.bfloat16).contiguous()
        keep += [beta, gamma]
        beta_ptr, gamma_ptr = beta.data_ptr(), gamma.data_ptr()
        epi = FCAI_EPI_IGDN if bool(getattr(gdn, "inverse", False)) else FCAI_EPI_GDN
    out_format = FCAI_FMT_NCHW_F32 if out_f32 else FCAI_FMT_NHWC_BF16
    desc = FcaiLayer(
        kind=FCAI_LAYER_DECONV5S2 if transposed else FCAI_LAYER_CONV5S2,
        cin=cin,
        cout=cout,
        npad=npad,
        epilogue=epi,
        in_format=FCAI_FMT_NCHW_F32 if first else FCAI_FMT_NHWC_BF16,
        out_format=out_format,
        clamp01=1 if clamp else 0,
        algorithm=FCAI_ALGO_SCATTER if scatter else (FCAI_ALGO_IMPLICIT_GEMM_PAIR if pair else FCAI_ALGO_IMPLICIT_GEMM),
        precision=FCAI_PREC_FP8_E4M3 if precision == "fp8" else FCAI_PREC_BF16,
        act_scale=None,
        weight_scale=w_scale,
        out_channel_offset=0,
        amax_out=None,
        out_channels_total=0,
        reserved=0,
        weight=weight.data_ptr(),
        bias=bias.data_ptr(),
        gdn_beta=beta_ptr,
        gdn_gamma=gamma_ptr,
    )
    return _Layer(desc, tuple(keep), desc.kind, cout, npad, out_format, precision=precision)


def _make_split_layer(conv: nn.Conv2d, *, clamp: bool, precision: str = "bf16") -> _Layer:
    """A convolution to fp32 NCHW with more output channels than one MMA
    takes (the 320-channel latent layer of FactorizedPrior(192, 320)): two
    halves of 160 channels, each its own launch on the same input, writing
    its channel range of the shared output.  FP8: both halves use the whole
    weight's per-tensor scale, as one scaled GEMM would."""
    cout = conv.out_channels
    if cout != 320:
        raise ConfigurationError("layers wider than 256 channels are built for the 320-channel latent "
                                 "(two launches of 160 channels)")
    width = cout // 2
    fp8_scale = fp8_weight_scale(conv.weight) if precision == "fp8" else None
    parts = []
    for c0 in range(0, cout, width):
        c1 = c0 + width
        sub = nn.Conv2d(conv.in_channels, c1 - c0, 5, 2, 2).to(conv.weight.device)
        with torch.no_grad():
            sub.weight.copy_(conv.weight[c0:c1])
            sub.bias.copy_(conv.bias[c0:c1])
        part = _make_layer(sub, None, first=False, out_f32=True, clamp=clamp, precision=precision,
                           fp8_scale=fp8_scale)
        part.desc.out_channel_offset = c0
        part.desc.out_channels_total = cout
        parts.append(part)
    return _Layer(None, (), FCAI_LAYER_CONV5S2, cout, parts[0].npad, FCAI_FMT_NCHW_F32, precision=precision,
                  parts=tuple(parts))


def _run(layers, x: torch.Tensor, first_is_nchw: bool) -> torch.Tensor:
    # The host issues these launches while the GPU runs the previous ones;
    # plain ints go to the native calls (their argtypes are declared).
    lib = _native.lib()
    forward = lib.fcai_layer_forward
    dev = x.device
    stream = _native.stream_handle(dev)
    launches = 0
    B = x.shape[0]
    if first_is_nchw:
        h, w = x.shape[2], x.shape[3]
    else:
        h, w = x.shape[1], x.shape[2]
    cur = x
    scal = None  # [scale, amax bits] of the current input when the producing layer computed its amax
    for i, layer in enumerate(layers):
        ho, wo = (2 * h, 2 * w) if layer.kind == FCAI_LAYER_DECONV5S2 else ((h - 1) // 2 + 1, (w - 1) // 2 + 1)
        # an FP8 next layer takes its input's amax from this layer's epilogue
        nxt = layers[i + 1] if i + 1 < len(layers) else None
        feeds_fp8 = (nxt is not None and nxt.precision == "fp8" and layer.out_format == FCAI_FMT_NHWC_BF16
                     and not layer.parts and layer.desc.algorithm != FCAI_ALGO_SCATTER)
        if layer.out_format == FCAI_FMT_NHWC_BF16:
            out = torch.empty((B, ho, wo, layer.npad), dtype=torch.bfloat16, device=dev)
        else:
            out = torch.empty((B, layer.cout, ho, wo), dtype=torch.float32, device=dev)
        timing = LAYER_TIMING
        if timing is not None:
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
        src = cur
        if layer.precision == "fp8":
            # the input's per-tensor e4m3 copy and its scale (amax / 448); the
            # amax came with the input when the previous layer produced it
            src = torch.empty(cur.shape, dtype=torch.uint8, device=dev)
            ready = scal is not None
            if not ready:
                scal = torch.zeros(2, dtype=torch.float32, device=dev)
            _native.check(lib.fcai_quantize_e4m3(cur.data_ptr(), src.data_ptr(), scal.data_ptr(), scal.data_ptr() + 4,
                                                 1 if ready else 0, cur.numel(), stream))
            launches += 1 if ready else 2
            for target in layer.parts or (layer,):
                target.desc.act_scale = scal.data_ptr()
        next_scal = None
        if layer.parts:
            for part in layer.parts:
                rc = forward(part.ref, B, h, w, src.data_ptr(), out.data_ptr(), None, stream)
                if rc:
                    _native.check(rc)
                launches += 1
        elif feeds_fp8:
            next_scal = torch.zeros(2, dtype=torch.float32, device=dev)
            layer.desc.amax_out = next_scal.data_ptr() + 4
            try:
                rc = forward(layer.ref, B, h, w, src.data_ptr(), out.data_ptr(), None, stream)
            finally:
                layer.desc.amax_out = None  # the buffer is this call's
            if rc:
                _native.check(rc)
            launches += 1
        else:
            rc = forward(layer.ref, B, h, w, src.data_ptr(), out.data_ptr(), None, stream)
            if rc:
                _native.check(rc)
            launches += 1
        scal = next_scal
        if timing is not None:
            ev1.record()
            timing.append((layer.name, layer.flops(B, h, w), ev0, ev1))
        cur, h, w = out, ho, wo
    _native.count_launches(launches)
    return cur


class _Packed(nn.Sequential):
    """A Sequential that keeps the FP32 child modules (so parameter names and
    state_dict keys do not change) and runs packed tensor-core layers built
    from them; the packs are rebuilt if a parameter is modified in place."""

    def _signature(self):
        # The children, and each parameter's identity and version counter
        # (inference tensors have none, and cannot change in place).  The
        # parameters are read from the dicts of the modules that own them,
        # collected again whenever a child is replaced: a walk through
        # parameters() on every call costs more than a layer launch.
        children = tuple(id(m) for m in self._modules.values())
        if getattr(self, "_owner_key", None) != children:
            self._owners = [m for m in self.modules() if m._parameters]
            self._owner_key = children
        sig = [children]
        for owner in self._owners:
            for t in owner._parameters.values():
                if t is not None:
                    sig.append((id(t), -1 if t.is_inference() else t._version))
        return tuple(sig)

    def _refresh_if_stale(self) -> None:
        if self._sig != self._signature():
            with torch.no_grad():
                self._build()
            self._sig = self._signature()


def resolve_precisions(prefix: str, modules: list, requested: Mapping[str, str] | None, *, first_conv: int | None,
                       last_f32: bool) -> tuple[list[str], list[tuple[str, str, str, str | None]]]:
    """Per fused layer of a 7-module g_a / g_s: the operand precision the B200
    kernels use ("bf16" or "fp8"), and per module (path, requested, applied,
    reason).  Convolutions requested in "fp8" get the e4m3 kernels where one
    exists; every other request runs with bf16 operands (a 16-bit format:
    "fp16" requests keep 16-bit operands, in bf16).  GDN / IGDN modules run
    inside the convolution kernel, whose norm GEMM is bf16."""
    requested = dict(requested or {})
    layer_prec, notes = [], []
    for i in range(0, 7, 2):
        conv = modules[i]
        gdn = modules[i + 1] if i + 1 < 7 else None
        path = f"{prefix}.{i}"
        want = requested.get(path, "bf16")
        applied, reason = "bf16", None
        if want == "fp8":
            reason = fp8_supported(conv, gdn, first=(i == first_conv), out_f32=(i == 6 and last_f32))
            if reason is None:
                applied = "fp8"
        elif want not in ("bf16", "fp16", "fp32"):
            raise ConfigurationError(f"unknown precision {want!r} for {path}")
        elif want != "bf16":
            reason = f"{want} runs with bf16 operands on the B200 kernels"
        layer_prec.append(applied)
        notes.append((path, want, applied, reason))
        if gdn is not None:
            gpath = f"{prefix}.{i + 1}"
            gwant = requested.get(gpath, "bf16")
            notes.append((gpath, gwant, "bf16",
                          None if gwant == "bf16" else "the fused GDN norm GEMM runs with bf16 operands"))
    return layer_prec, notes


class B200Analysis(_Packed):
    """g_a on the tensor cores: fp32 NCHW image -> fp32 NCHW latent.

    ``precisions`` maps module paths ("g_a.0" ... "g_a.6") to requested
    precisions (a saved precision map); see ``resolve_precisions``."""

    def __init__(self, g_a: nn.Sequential, precisions: Mapping[str, str] | None = None):
        super().__init__(*list(g_a))
        if len(self) != 7:
            raise ConfigurationError("g_a must be conv, GDN, conv, GDN, conv, GDN, conv")
        self._layer_prec, self.precision_notes = resolve_precisions("g_a", list(self), precisions, first_conv=0,
                                                                     last_f32=True)
        self._build()
        self._sig = self._signature()

    def _build(self) -> None:
        m = list(self)
        lp = self._layer_prec
        self._layers = [
            _make_layer(m[0], m[1], first=True, out_f32=False, clamp=False, precision=lp[0]),
            _make_layer(m[2], m[3], first=False, out_f32=False, clamp=False, precision=lp[1]),
            _make_layer(m[4], m[5], first=False, out_f32=False, clamp=False, precision=lp[2]),
            _make_layer(m[6], None, first=False, out_f32=True, clamp=False, precision=lp[3]),
        ]
        for i, layer in enumerate(self._layers):
            layer.name = f"g_a.{2 * i}" + ("+gdn" if i < 3 else "")

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda or x.dim() != 4 or x.shape[1] != 3:
            raise ValueError("B200Analysis expects a CUDA [B, 3, H, W] tensor")
        self._refresh_if_stale()
        x = x.float().contiguous()
        with _native.on_device(x.device):
            return _run(self._layers, x, first_is_nchw=True)


class B200Synthesis(_Packed):
    """g_s on the tensor cores: fp32 NCHW latent -> fp32 NCHW image.

    ``forward(y, clamp=True)`` applies the final clamp to [0, 1] inside the
    last layer (the codec's ``g_s(y_hat).clamp_(0, 1)``)."""

    fuses_clamp = True

    def __init__(self, g_s: nn.Sequential, precisions: Mapping[str, str] | None = None):
        super().__init__(*list(g_s))
        if len(self) != 7:
            raise ConfigurationError("g_s must be deconv, IGDN, deconv, IGDN, deconv, IGDN, deconv")
        self.channels = self[0].in_channels
        self._layer_prec, self.precision_notes = resolve_precisions("g_s", list(self), precisions, first_conv=None,
                                                                     last_f32=True)
        self._build()
        self._sig = self._signature()

    def _build(self) -> None:
        m = list(self)
        lp = self._layer_prec
        self._layers = [
            _make_layer(m[0], m[1], first=False, out_f32=False, clamp=False, precision=lp[0]),
            _make_layer(m[2], m[3], first=False, out_f32=False, clamp=False, precision=lp[1]),
            _make_layer(m[4], m[5], first=False, out_f32=False, clamp=False, precision=lp[2]),
        ]
        self._last = _make_layer(m[6], None, first=False, out_f32=True, clamp=False, precision=lp[3])
        self._last_clamped = _make_layer(m[6], None, first=False, out_f32=True, clamp=True, precision=lp[3])
        for i, layer in enumerate(self._layers):
            layer.name = f"g_s.{2 * i}+igdn"
        self._last.name = self._last_clamped.name = "g_s.6"

    def forward(self, y: torch.Tensor, clamp: bool = False) -> torch.Tensor:
        if not y.is_cuda or y.dim() != 4 or y.shape[1] != self.channels:
            raise ValueError("B200Synthesis expects a CUDA [B, M, h, w] tensor")
        self._refresh_if_stale()
        y = y.float().contiguous()
        B, C, h, w = y.shape
        with _native.on_device(y.device):
            nhwc = torch.empty((B, h, w, C), dtype=torch.bfloat16, device=y.device)
            stream = _native.stream_handle(y.device)
            _native.check(_native.lib().fcai_nchw_f32_to_nhwc_bf16(y.data_ptr(), nhwc.data_ptr(), B, C, h, w, stream))
            _native.count_launches(1)
            return _run(self._layers + [self._last_clamped if clamp else self._last], nhwc, first_is_nchw=False)


def convert_factorized_prior(model: nn.Module, precision: str = "bf16",
                             layer_precisions: Mapping[str, str] | None = None) -> nn.Module:
    """Swap g_a / g_s for the B200 tensor-core modules (in place; returns the model).

    ``layer_precisions`` (module path -> "fp8" / "fp16" / "bf16" / "fp32",
    e.g. a loaded precision map) selects the e4m3 kernels per convolution
    where they exist; the modules' ``precision_notes`` record what ran.
    ``precision="fp8"`` without a map requests e4m3 for every convolution
    (those without an e4m3 kernel run bf16 and say why)."""
    if precision not in ("bf16", "fp8"):
        raise ConfigurationError(f"unsupported transform precision {precision!r}")
    if precision == "fp8" and layer_precisions is None:
        layer_precisions = {f"{t}.{i}": "fp8" for t in ("g_a", "g_s") for i in (0, 2, 4, 6)}
    if not torch.cuda.is_available():
        raise ConfigurationError("B200 transforms require CUDA")
    dev = next(model.parameters()).device
    if dev.type != "cuda":
        raise ConfigurationError("convert the model after moving it to the CUDA device")
    with torch.no_grad(), torch.cuda.device(dev):
        g_a = B200Analysis(model.g_a, layer_precisions)
        g_s = B200Synthesis(model.g_s, layer_precisions)
    # the new modules hold the same FP32 children, so state_dict keys are unchanged
    model.g_a = g_a
    model.g_s = g_s
    return model
