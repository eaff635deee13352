"""Generate the per-layer golden vectors of the reference's BF16 operators.

The reference's BF16 transform path (``backends/pytorch/bf16_operators.py``:
``BF16Conv2d``, ``BF16ConvTranspose2d``, ``BF16GDN``) is loaded from its
checkout by file path (it imports only torch) and run on the CPU, layer by
layer, over this repository's FactorizedPrior(128, 192) built from a fixed
seed (GDN gamma perturbed off the diagonal, so the GDN GEMM mixes channels).
Each layer's input is the previous reference layer's output, and every
stored tensor is bf16-valued, kept as its exact 16-bit pattern.  The
fixture pins the tcgen05 layers to the reference's definition of its BF16
path (tests/test_bf16_golden_gpu.py).  The checkout is ``$FCAI_REFERENCE``,
else the ``reference_path`` that BASELINE.json records.

    python tests/golden/make_bf16_golden.py --out tests/golden/transforms/bf16_layers.npz
"""

from __future__ import annotations

import argparse
import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
for p in (ROOT, ROOT / "fast-compressai_b200"):
    sys.path.insert(0, str(p))

from oracle import build_ref  # noqa: E402
from tests.bf16_golden_model import IMAGE_SHAPE, LATENT_SHAPE, golden_model, layers, weight_checksum  # noqa: E402


def _load_reference_operators():
    root = build_ref.reference_root()
    if root is None:
        raise SystemExit("reference checkout not found ($FCAI_REFERENCE or BASELINE.json reference_path)")
    path = Path(root) / "src" / "fast_compressai" / "backends" / "pytorch" / "bf16_operators.py"
    spec = importlib.util.spec_from_file_location("reference_bf16_operators", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _ref_layer(ops, conv, gdn):
    """The reference's BF16 modules for one fused layer, built by its own factories."""
    if isinstance(conv, torch.nn.ConvTranspose2d):
        c = ops.conv_transpose2d_factory(conv, {})
    else:
        c = ops.conv2d_factory(conv, {})
    c.load_state_dict(conv.state_dict())
    g = ops.gdn_factory(gdn, {}) if gdn is not None else None
    return c, g


def _bits(t: torch.Tensor) -> np.ndarray:
    b = t.detach().to(torch.bfloat16).contiguous()
    assert torch.equal(b.float(), t.detach().float()), "reference output is not bf16-valued"
    return b.view(torch.int16).numpy().view(np.uint16)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(ROOT / "tests" / "golden" / "transforms" / "bf16_layers.npz"))
    args = ap.parse_args()
    ops = _load_reference_operators()
    model = golden_model()
    g = torch.Generator().manual_seed(11)
    x = torch.rand(IMAGE_SHAPE, generator=g)
    y_in = torch.round(torch.randn(LATENT_SHAPE, generator=g) * 4)
    out = {"weight_checksum": np.float64(weight_checksum(model)), "x": x.numpy(), "y_hat": y_in.numpy()}
    with torch.no_grad():
        for chain, cur in (("g_a", x), ("g_s", y_in)):
            for i, (conv, gdn) in enumerate(layers(model, chain)):
                c, gm = _ref_layer(ops, conv, gdn)
                cur = c(cur)
                if gm is not None:
                    cur = gm(cur)
                out[f"{chain}.{i}"] = _bits(cur)
    np.savez_compressed(args.out, **out)
    print({k: v.shape for k, v in out.items() if hasattr(v, "shape")})


if __name__ == "__main__":
    main()
