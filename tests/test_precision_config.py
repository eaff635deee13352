"""Saved precision maps on the CPU: the reference's schema-4 loader rules and
the mapping of a map onto the B200 transform layers (which modules get the
e4m3 kernels and why the others do not)."""

from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch

from fast_compressai.balle import FactorizedPrior
from fast_compressai.configs import PrecisionConfig, PrecisionConfigError, model_fingerprint
from fast_compressai.transforms import fp8_supported, resolve_precisions

FIXTURE = Path(__file__).parent / "golden" / "precision_map_factorized.json"


def _data():
    return json.loads(FIXTURE.read_text())


def test_fixture_loads_and_round_trips(tmp_path):
    config = PrecisionConfig.load(FIXTURE)
    assert config.coder == "warp_div" and config.p_ch == 16 and len(config.assignments) == 14
    prec = config.precision_by_path()
    assert prec["g_a.2"] == "fp8" and prec["g_a.0"] == "fp16" and prec["g_s.1"] == "fp8"
    again = PrecisionConfig.from_json(config.to_json())
    assert again == config
    out = config.save(tmp_path / "sub" / "map.json")
    assert PrecisionConfig.load(out) == config


@pytest.mark.parametrize("mutate,message", [
    (lambda d: d.update(schema_version=3), "unsupported precision config schema"),
    (lambda d: d.pop("epsilon"), "missing or unknown fields"),
    (lambda d: d.update(extra=1), "missing or unknown fields"),
    (lambda d: d.update(kind="other"), "invalid precision config kind"),
    (lambda d: d.update(model_fingerprint="xyz"), "model_fingerprint must be a SHA-256 hex digest"),
    (lambda d: d.update(rd_cost_formula="psnr"), "unsupported RD Cost formula"),
    (lambda d: d.update(epsilon=-1.0), "epsilon and profile cost must be non-negative"),
    (lambda d: d.update(p_ch=0), "p_ch must be a positive integer or None"),
    (lambda d: d.update(device_capability=[9]), "device_capability must be an integer pair"),
    (lambda d: d["assignments"].append(dict(d["assignments"][0])), "duplicate module paths"),
    (lambda d: d["assignments"][0].update(precision=""), "assignment precision must be non-empty"),
    (lambda d: d["assignments"][0].update(probe_rd_cost=float("inf")), "probe_rd_cost must be finite"),
])
def test_loader_rejections(mutate, message):
    data = _data()
    mutate(data)
    with pytest.raises(PrecisionConfigError, match=message):
        PrecisionConfig.from_json(json.dumps(data))
    with pytest.raises(PrecisionConfigError, match="not valid JSON"):
        PrecisionConfig.from_json("{")


def test_compatibility_check_names_the_mismatches():
    config = PrecisionConfig.load(FIXTURE)
    config.validate_compatibility(coder="warp_div", p_ch=16)
    with pytest.raises(PrecisionConfigError, match="incompatible: coder, p_ch"):
        config.validate_compatibility(coder="rans", p_ch=4)


def test_model_fingerprint_follows_the_weights():
    torch.manual_seed(0)
    a = FactorizedPrior(8, 12)
    b = FactorizedPrior(8, 12)
    b.load_state_dict(a.state_dict())
    assert model_fingerprint(a) == model_fingerprint(b)
    with torch.no_grad():
        b.g_a[0].weight[0, 0, 0, 0] += 1.0
    assert model_fingerprint(a) != model_fingerprint(b)


def test_fixture_map_on_the_b200_layers():
    # FactorizedPrior(128, 192): of the map's fp8 convolutions, g_a.2 (128 -> 128
    # + GDN) and g_a.6 (128 -> 192 latent) have e4m3 kernels; every GDN runs
    # inside its convolution with a bf16 norm GEMM; fp16 modules run bf16
    model = FactorizedPrior(128, 192)
    prec = PrecisionConfig.load(FIXTURE).precision_by_path()
    lp_a, notes_a = resolve_precisions("g_a", list(model.g_a), prec, first_conv=0, last_f32=True)
    lp_s, notes_s = resolve_precisions("g_s", list(model.g_s), prec, first_conv=None, last_f32=True)
    assert lp_a == ["bf16", "fp8", "bf16", "fp8"]
    assert lp_s == ["bf16", "bf16", "bf16", "bf16"]
    notes = {path: (want, got, why) for path, want, got, why in notes_a + notes_s}
    assert notes["g_a.2"] == ("fp8", "fp8", None) and notes["g_a.6"] == ("fp8", "fp8", None)
    assert notes["g_a.1"][:2] == ("fp8", "bf16") and "norm GEMM" in notes["g_a.1"][2]
    assert notes["g_a.0"][:2] == ("fp16", "bf16") and "bf16 operands" in notes["g_a.0"][2]
    assert len(notes) == 14


def test_fp8_kernel_coverage_rules():
    model = FactorizedPrior(128, 192)
    g_a, g_s = list(model.g_a), list(model.g_s)
    assert fp8_supported(g_a[0], g_a[1], first=True, out_f32=False) is not None  # cin = 3
    assert fp8_supported(g_a[2], g_a[3], first=False, out_f32=False) is None
    # cin = 192: two 128-channel K blocks, the second half zero-filled by TMA
    assert fp8_supported(g_s[0], g_s[1], first=False, out_f32=False) is None
    assert fp8_supported(g_s[2], g_s[3], first=False, out_f32=False) is None
    assert fp8_supported(g_s[6], None, first=False, out_f32=True) is not None  # scatter layer
    assert fp8_supported(g_a[6], None, first=False, out_f32=True) is None
    # FactorizedPrior(192, 320): 192-channel GDN / IGDN, the split 320-channel latent, g_s.0 (cin = 320)
    big = FactorizedPrior(192, 320)
    b_a, b_s = list(big.g_a), list(big.g_s)
    assert fp8_supported(b_a[2], b_a[3], first=False, out_f32=False) is None
    assert fp8_supported(b_a[6], None, first=False, out_f32=True) is None
    assert fp8_supported(b_s[0], b_s[1], first=False, out_f32=False) is None
    assert fp8_supported(b_s[4], b_s[5], first=False, out_f32=False) is None
    assert fp8_supported(b_a[0], b_a[1], first=True, out_f32=False) is not None
    odd = torch.nn.Conv2d(96, 128, 5, 2, 2)
    assert "multiple of 64" in fp8_supported(odd, None, first=False, out_f32=False)
    with pytest.raises(Exception, match="unknown precision"):
        resolve_precisions("g_a", g_a, {"g_a.2": "int4"}, first_conv=0, last_f32=True)
