"""FP32 FactorizedPrior model (bmshj2018-factorized architecture).

CompressAI is not installed in this build's environments, so the package
ships its own FP32 model with the same architecture and the same attribute
surface the reference's codec uses (``g_a``, ``g_s``, ``entropy_bottleneck``
with ``_quantized_cdf``, ``_cdf_length``, ``_offset``, ``_get_medians``,
``_extend_ndims``, ``_build_indexes``, ``quantize``, ``dequantize``,
``update``), written from the published papers:

* transforms: Balle, Minnen, Singh, Hwang, Johnston, "Variational image
  compression with a scale hyperprior", ICLR 2018 (factorized-prior
  baseline): four 5x5 stride-2 convolutions with GDN between them, and the
  mirrored transposed convolutions with inverse GDN;
* GDN: Balle, Laparra, Simoncelli, "Density modeling of images using a
  generalized normalization transformation", ICLR 2016,
  ``y_i = x_i / sqrt(beta_i + sum_j gamma_ij x_j^2)``, parameters kept
  non-negative by the squared, lower-bounded parametrisation of Balle et al.
  "End-to-end optimized image compression", ICLR 2017;
* entropy model: the univariate non-parametric density of the 2018 paper
  (appendix 6.1): per channel a monotone cumulative
  ``c(x) = sigmoid(f_K(...f_1(x)))`` with ``f_k(x) = h_k(H_k x + b_k)``,
  ``h_k(x) = x + tanh(a_k) * tanh(x)`` and ``H_k = softplus(raw_k)``.

The 16-bit CDF quantisation in ``update`` is this package's own (every
symbol keeps a frequency of at least 1, frequencies sum to 2^16, the last
symbol is the escape/tail symbol); it is not CompressAI's routine, so
tables differ from a CompressAI model with the same weights.  The coder
itself is defined for any valid table, which is what parity is judged on.
"""

from __future__ import annotations

import math

import numpy as np
import torch
from torch import nn
from torch.nn import functional as F

CDF_PRECISION = 16


class NonNegative(nn.Module):
    """Stores v >= bound as p = sqrt(v + pedestal); reads lower_bound(p)^2 - pedestal."""

    def __init__(self, minimum: float = 0.0, reparam_offset: float = 2.0 ** -18):
        super().__init__()
        self.minimum = float(minimum)
        self.reparam_offset = float(reparam_offset)
        self.register_buffer("pedestal", torch.tensor(reparam_offset ** 2), persistent=False)
        self.register_buffer("lower", torch.tensor(math.sqrt(self.minimum + reparam_offset ** 2)), persistent=False)

    def init(self, value: torch.Tensor) -> torch.Tensor:
        return torch.sqrt(torch.clamp(value + self.pedestal, min=float(self.pedestal)))

    def forward(self, p: torch.Tensor) -> torch.Tensor:
        bounded = torch.maximum(p, self.lower.to(p.dtype))
        return bounded * bounded - self.pedestal.to(p.dtype)


class GDN(nn.Module):
    """Generalized divisive normalization (inverse=True gives IGDN)."""

    def __init__(self, in_channels: int, inverse: bool = False, beta_min: float = 1e-6, gamma_init: float = 0.1):
        super().__init__()
        self.inverse = bool(inverse)
        self.beta_reparam = NonNegative(minimum=beta_min)
        self.gamma_reparam = NonNegative()
        self.beta = nn.Parameter(self.beta_reparam.init(torch.ones(in_channels)))
        self.gamma = nn.Parameter(self.gamma_reparam.init(gamma_init * torch.eye(in_channels)))

    def effective_params(self) -> tuple[torch.Tensor, torch.Tensor]:
        """(beta [C], gamma [C, C]) after the non-negative parametrisation."""
        return self.beta_reparam(self.beta), self.gamma_reparam(self.gamma)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        beta, gamma = self.effective_params()
        c = beta.numel()
        norm = F.conv2d(x * x, gamma.reshape(c, c, 1, 1), beta)
        return x * (torch.sqrt(norm) if self.inverse else torch.rsqrt(norm))


def _conv(cin: int, cout: int) -> nn.Conv2d:
    return nn.Conv2d(cin, cout, kernel_size=5, stride=2, padding=2)


def _deconv(cin: int, cout: int) -> nn.ConvTranspose2d:
    return nn.ConvTranspose2d(cin, cout, kernel_size=5, stride=2, padding=2, output_padding=1)


class EntropyBottleneck(nn.Module):
    """Factorized (per-channel, non-parametric) latent density with 16-bit CDF tables."""

    def __init__(self, channels: int, tail_mass: float = 1e-9, init_scale: float = 10.0,
                 filters: tuple[int, ...] = (3, 3, 3)):
        super().__init__()
        self.channels = int(channels)
        self.tail_mass = float(tail_mass)
        self.init_scale = float(init_scale)
        self.filters = tuple(int(f) for f in filters)
        dims = (1,) + self.filters + (1,)
        # spread init_scale over the layers so the initial cumulative spans ~[-init_scale, init_scale]
        per_layer = self.init_scale ** (1.0 / (len(self.filters) + 1))
        self._raw_matrices = nn.ParameterList()
        self._biases = nn.ParameterList()
        self._raw_factors = nn.ParameterList()
        for i in range(len(dims) - 1):
            init = math.log(math.expm1(1.0 / per_layer / dims[i + 1]))
            self._raw_matrices.append(nn.Parameter(torch.full((channels, dims[i + 1], dims[i]), init)))
            self._biases.append(nn.Parameter(torch.rand(channels, dims[i + 1], 1) - 0.5))
            if i < len(dims) - 2:
                self._raw_factors.append(nn.Parameter(torch.zeros(channels, dims[i + 1], 1)))
        q = torch.tensor([-self.init_scale, 0.0, self.init_scale])
        self.quantiles = nn.Parameter(q.repeat(channels, 1, 1))
        self.register_buffer("_offset", torch.zeros(0, dtype=torch.int32))
        self.register_buffer("_quantized_cdf", torch.zeros(0, dtype=torch.int32))
        self.register_buffer("_cdf_length", torch.zeros(0, dtype=torch.int32))

    # -- density ---------------------------------------------------------
    def _logits_cumulative(self, x: torch.Tensor) -> torch.Tensor:
        """x: [C, 1, S] -> pre-sigmoid cumulative [C, 1, S]."""
        h = x
        n = len(self._raw_matrices)
        for i in range(n):
            h = torch.matmul(F.softplus(self._raw_matrices[i]), h) + self._biases[i]
            if i < n - 1:
                h = h + torch.tanh(self._raw_factors[i]) * torch.tanh(h)
        return h

    def likelihood(self, y: torch.Tensor) -> torch.Tensor:
        """P(round(y) = y) for integer-valued y [B, C, ...] relative to the medians."""
        c = self.channels
        v = y.transpose(0, 1).reshape(c, 1, -1)
        lo = self._logits_cumulative(v - 0.5)
        hi = self._logits_cumulative(v + 0.5)
        s = -torch.sign(lo + hi)
        p = torch.abs(torch.sigmoid(s * hi) - torch.sigmoid(s * lo))
        shape = (y.shape[1], y.shape[0], *y.shape[2:])
        return p.reshape(shape).transpose(0, 1)

    # -- coder interface used by the codec --------------------------------
    def _get_medians(self) -> torch.Tensor:
        return self.quantiles[:, 0, 1]

    @staticmethod
    def _extend_ndims(tensor: torch.Tensor, n: int) -> torch.Tensor:
        return tensor.reshape(tensor.shape + (1,) * n)

    def _build_indexes(self, size, device=None) -> torch.Tensor:
        size = tuple(int(s) for s in size)
        if len(size) < 2 or size[1] != self.channels:
            raise ValueError("index shape must be [B, channels, ...]")
        idx = torch.arange(self.channels, dtype=torch.int32, device=device)
        idx = idx.reshape((1, -1) + (1,) * (len(size) - 2))
        return idx.expand(size).contiguous()

    @staticmethod
    def quantize(inputs: torch.Tensor, mode: str, means: torch.Tensor | None = None) -> torch.Tensor:
        if mode == "noise":
            return inputs + torch.empty_like(inputs).uniform_(-0.5, 0.5)
        shifted = inputs if means is None else inputs - means
        rounded = torch.round(shifted)
        if mode == "symbols":
            return rounded.int()
        if mode == "dequantize":
            return rounded if means is None else rounded + means
        raise ValueError(f'invalid quantization mode "{mode}"')

    @staticmethod
    def dequantize(inputs: torch.Tensor, means: torch.Tensor | None = None, dtype=torch.float) -> torch.Tensor:
        out = inputs.type(dtype)
        return out if means is None else out + means

    @torch.no_grad()
    def update(self, force: bool = False) -> bool:
        """Build the 16-bit CDF tables from the current density."""
        if self._offset.numel() > 0 and not force:
            return False
        q = self.quantiles.detach()
        medians = q[:, 0, 1]
        below = torch.ceil(medians - q[:, 0, 0]).clamp(min=0).to(torch.int64)
        above = torch.ceil(q[:, 0, 2] - medians).clamp(min=0).to(torch.int64)
        lengths = (below + above + 1)
        width = int(lengths.max())
        start = (medians - below.to(medians.dtype)).reshape(-1, 1, 1)
        grid = start + torch.arange(width, dtype=medians.dtype, device=medians.device).reshape(1, 1, -1)
        lo = self._logits_cumulative(grid - 0.5)
        hi = self._logits_cumulative(grid + 0.5)
        s = -torch.sign(lo + hi)
        pmf = torch.abs(torch.sigmoid(s * hi) - torch.sigmoid(s * lo))[:, 0, :]
        tails = torch.sigmoid(lo[:, 0, :1]) + torch.sigmoid(-hi[:, 0, -1:])
        cdfs = quantize_cdfs(pmf.double().cpu().numpy(), tails[:, 0].double().cpu().numpy(), lengths.cpu().numpy())
        dev = self.quantiles.device
        self._quantized_cdf = torch.from_numpy(cdfs).to(dev)
        self._cdf_length = (lengths + 2).to(torch.int32).to(dev)
        self._offset = (-below).to(torch.int32).to(dev)
        return True


def quantize_cdfs(pmf: np.ndarray, tail: np.ndarray, lengths: np.ndarray) -> np.ndarray:
    """Integer CDF rows [C, max(lengths) + 2] at 16-bit precision.

    Row c holds lengths[c] + 1 symbol frequencies (the pmf, then the tail
    mass as the escape symbol), each >= 1 and summing to 2^16, as a
    cumulative table starting at 0; unused entries are 0."""
    total = 1 << CDF_PRECISION
    C = pmf.shape[0]
    out = np.zeros((C, int(lengths.max()) + 2), dtype=np.int32)
    for c in range(C):
        n = int(lengths[c])
        p = np.concatenate([np.clip(pmf[c, :n], 0.0, None), [max(float(tail[c]), 0.0)]])
        s = p.sum()
        p = p / s if s > 0 else np.full(n + 1, 1.0 / (n + 1))
        freq = np.maximum(1, np.floor(p * total + 0.5)).astype(np.int64)
        excess = int(freq.sum()) - total
        while excess != 0:
            order = np.argsort(-freq, kind="stable")
            if excess < 0:
                freq[order[0]] += -excess
                excess = 0
            else:
                for j in order:
                    if excess == 0:
                        break
                    take = min(excess, int(freq[j]) - 1)
                    freq[j] -= take
                    excess -= take
        out[c, 1:n + 2] = np.cumsum(freq)
    return out


class FactorizedPrior(nn.Module):
    """bmshj2018-factorized: g_a / g_s transforms with a factorized entropy bottleneck."""

    def __init__(self, N: int, M: int):
        super().__init__()
        self.N = int(N)
        self.M = int(M)
        self.entropy_bottleneck = EntropyBottleneck(M)
        self.g_a = nn.Sequential(_conv(3, N), GDN(N), _conv(N, N), GDN(N), _conv(N, N), GDN(N), _conv(N, M))
        self.g_s = nn.Sequential(
            _deconv(M, N), GDN(N, inverse=True), _deconv(N, N), GDN(N, inverse=True), _deconv(N, N),
            GDN(N, inverse=True), _deconv(N, 3),
        )

    @property
    def downsampling_factor(self) -> int:
        return 16

    def update(self, scale_table=None, force: bool = False) -> bool:
        del scale_table
        return self.entropy_bottleneck.update(force=force)

    def forward(self, x: torch.Tensor) -> dict:
        y = self.g_a(x)
        medians = self.entropy_bottleneck._extend_ndims(self.entropy_bottleneck._get_medians(), y.ndim - 2)
        y_hat = self.entropy_bottleneck.quantize(y, "dequantize", medians)
        likelihoods = self.entropy_bottleneck.likelihood(y_hat - medians)
        return {"x_hat": self.g_s(y_hat), "likelihoods": {"y": likelihoods}}

    def compress(self, x: torch.Tensor):
        raise NotImplementedError(
            "FactorizedPrior.compress here has no CPU RANS coder; use fast_compressai.accelerate(model, P=...) "
            "for the warp_div GPU path"
        )

    def decompress(self, strings, shape):
        raise NotImplementedError(
            "FactorizedPrior.decompress here has no CPU RANS coder; use the accelerated model's decompress"
        )
