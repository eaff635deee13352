"""Build the reference's own warp_div CUDA extension from its sources, for sm_100a.

TEST INFRASTRUCTURE ONLY (the parity checker of the GPU tests and of the
golden fixtures).  Sources are compiled where they lie in the reference
checkout: $FCAI_REFERENCE, else the ``reference_path`` that BASELINE.json at
the repository root records.  Nothing is copied into this repository.  Output: oracle/_ref/_warp_div_ref.so, a torch
extension exposing the reference's pybind entry points ``encode_warp_div``
and ``decode_warp_div`` (coders/cuda/ans_gpu.cpp:25-30).

    python oracle/build_ref.py          # in a container that has the reference
"""

from __future__ import annotations

import importlib.util
import json
import os
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
NAME = "_warp_div_ref"
SOURCES = ["ans_gpu.cpp", "warp_ans_kernel.cu", "warp_ans_kernel_v2.cu", "warp_index_check.cu"]


def reference_root() -> Path | None:
    env = os.environ.get("FCAI_REFERENCE")
    if env:
        return Path(env)
    try:
        rec = json.loads((HERE.parent / "BASELINE.json").read_text())
    except (OSError, ValueError):
        return None
    path = rec.get("reference_path")
    return Path(path) if path else None


def built_path() -> Path:
    return OUT / f"{NAME}.so"


def build(force: bool = False) -> Path | None:
    """Compile the reference extension if its sources are present; returns the .so path."""
    root = reference_root()
    src_dir = root / "src" / "fast_compressai" / "coders" / "cuda" if root else None
    if src_dir is None or not src_dir.is_dir():
        return built_path() if built_path().exists() else None
    if built_path().exists() and not force:
        return built_path()
    from torch.utils import cpp_extension

    OUT.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    cpp_extension.load(
        name=NAME,
        sources=[str(src_dir / s) for s in SOURCES],
        extra_cflags=["-O2"],
        extra_cuda_cflags=["-O3", "-gencode", "arch=compute_100a,code=sm_100a"],
        build_directory=str(OUT),
        with_cuda=True,
        is_python_module=True,
        verbose=False,
    )
    # keep only the module; object files and ninja logs stay out of the tree
    for p in OUT.iterdir():
        if p.name != f"{NAME}.so":
            if p.is_dir():
                shutil.rmtree(p)
            else:
                p.unlink()
    return built_path()


def load():
    """Import the built reference extension (no sources needed)."""
    path = built_path()
    if not path.exists():
        raise FileNotFoundError(f"{path} is not built (run oracle/build_ref.py where the reference is present)")
    import torch  # noqa: F401  (the extension links against torch)

    spec = importlib.util.spec_from_file_location(NAME, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
