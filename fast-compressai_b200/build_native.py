"""Build the package's native library (CUDA kernels + C ABI) for sm_100a.

    python fast-compressai_b200/build_native.py [--force]

Produces fast_compressai/_lib/libfcai_b200.so in-tree with nvcc
(``-gencode arch=compute_100a,code=sm_100a``).  No GPU is needed to build.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent
CSRC = ROOT / "csrc"
INCLUDE = ROOT.parent / "include"
LIB_DIR = ROOT / "fast_compressai" / "_lib"
LIB = LIB_DIR / "libfcai_b200.so"

SOURCES = [
    "warp_div.cu",
    "conv_tc.cu",
]
HEADERS = ["fcai_common.h", "tc_ptx.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build fast_compressai")


def _inputs() -> list[Path]:
    files = [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS]
    files += sorted(INCLUDE.glob("*.h"))
    return files


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _inputs())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    nvcc = _nvcc()
    objdir = ROOT / "_build"
    objdir.mkdir(exist_ok=True)
    objs = []
    for src in SOURCES:
        obj = objdir / (Path(src).stem + ".o")
        cmd = [nvcc, *ARCH, *FLAGS, "-I", str(INCLUDE), "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(f".so.{os.getpid()}.tmp")
    cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *objs]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args(argv)
    print(build(force=args.force, verbose=True))
    return 0


if __name__ == "__main__":
    sys.exit(main())
