"""Host-side rules of the B200 transform modules that need no GPU: the
parameter-version check that rebuilds the packed layers, the split of a
320-channel latent layer into two 160-channel launches (with one FP8 weight
scale), and the accepted transform precisions."""

from __future__ import annotations

import pytest
import torch
from torch import nn

from fast_compressai import accelerate
from fast_compressai.balle import FactorizedPrior
from fast_compressai.config import ConfigurationError
from fast_compressai.transforms import (FCAI_FMT_NCHW_F32, FCAI_PREC_FP8_E4M3, _make_layer, _Packed,
                                        fp8_weight_scale)


class _Probe(_Packed):
    """A _Packed whose build only counts (no native layers)."""

    def __init__(self, modules):
        super().__init__(*modules)
        self.builds = 0
        self._build()
        self._sig = self._signature()

    def _build(self) -> None:
        self.builds += 1


def _probe():
    torch.manual_seed(0)
    return _Probe([nn.Conv2d(3, 8, 5, 2, 2), nn.Conv2d(8, 8, 5, 2, 2)])


def test_unchanged_parameters_keep_the_packs():
    m = _probe()
    for _ in range(3):
        m._refresh_if_stale()
    assert m.builds == 1


def test_in_place_edit_rebuilds_once():
    m = _probe()
    with torch.no_grad():
        m[0].weight.add_(1.0)
    m._refresh_if_stale()
    m._refresh_if_stale()
    assert m.builds == 2


def test_replaced_parameter_and_child_rebuild():
    m = _probe()
    m[1].bias = nn.Parameter(torch.zeros(8))
    m._refresh_if_stale()
    assert m.builds == 2
    m[1] = nn.Conv2d(8, 8, 5, 2, 2)  # a new child: its parameters are tracked from now on
    m._refresh_if_stale()
    assert m.builds == 3
    with torch.no_grad():
        m[1].weight.mul_(2.0)
    m._refresh_if_stale()
    assert m.builds == 4


def test_inference_tensors_have_no_version_to_compare():
    with torch.inference_mode():
        m = _probe()
        m._refresh_if_stale()
    assert m.builds == 1


def test_latent_wider_than_one_mma_is_split_in_two_halves():
    torch.manual_seed(1)
    conv = nn.Conv2d(192, 320, 5, 2, 2)
    layer = _make_layer(conv, None, first=False, out_f32=True, clamp=False)
    assert layer.desc is None and len(layer.parts) == 2 and layer.cout == 320
    assert [p.desc.out_channel_offset for p in layer.parts] == [0, 160]
    assert all(p.desc.out_channels_total == 320 and p.desc.cout == 160 and p.npad == 160 for p in layer.parts)
    assert all(p.out_format == FCAI_FMT_NCHW_F32 for p in layer.parts)
    # the halves hold the two channel ranges of the weight (packed [25][npad][cin])
    w0 = layer.parts[0].keep[0].float()
    ref = conv.weight.detach()[:160].permute(2, 3, 0, 1).reshape(25, 160, 192)
    assert torch.equal(w0, ref.to(torch.bfloat16).float())
    fp8 = _make_layer(conv, None, first=False, out_f32=True, clamp=False, precision="fp8")
    scales = {p.desc.weight_scale for p in fp8.parts}
    assert len(scales) == 1 and scales.pop() == pytest.approx(fp8_weight_scale(conv.weight), rel=0, abs=0)
    assert all(p.desc.precision == FCAI_PREC_FP8_E4M3 for p in fp8.parts) and fp8.precision == "fp8"


def test_other_wide_layers_are_refused():
    with pytest.raises(ConfigurationError, match="320-channel latent"):
        _make_layer(nn.Conv2d(192, 384, 5, 2, 2), None, first=False, out_f32=True, clamp=False)


def test_transform_precisions():
    model = FactorizedPrior(8, 12)
    with pytest.raises(ConfigurationError, match="transforms must be one of"):
        accelerate(model, P=4, coder="warp_div", transforms="int8")
