"""The C ABI from plain C (tests/native/c_abi_roundtrip.c): the header compiles
as C99 with every warning an error and the program links against the library
and the CUDA runtime alone (CPU); on a GPU the program's encode, pack and
checked and unchecked decodes return its symbols (no Python in that process).
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
LIB_DIR = ROOT / "fast-compressai_b200" / "fast_compressai" / "_lib"
CUDA = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
SRC = ROOT / "tests" / "native" / "c_abi_roundtrip.c"


def _build(out: Path) -> Path:
    if shutil.which("gcc") is None or not (CUDA / "include" / "cuda_runtime.h").exists():
        pytest.skip("gcc or the CUDA headers are not installed")
    exe = out / "c_abi_roundtrip"
    cmd = ["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-O2", f"-I{ROOT / 'include'}", f"-I{CUDA / 'include'}",
           str(SRC), "-o", str(exe), f"-L{LIB_DIR}", "-lfcai_b200", f"-L{CUDA / 'lib64'}", "-lcudart",
           f"-Wl,-rpath,{LIB_DIR}:{CUDA / 'lib64'}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_c_abi_program_compiles_and_links(tmp_path):
    assert _build(tmp_path).exists()


@pytest.mark.gpu
def test_c_abi_round_trip_without_python(tmp_path, cuda_device):
    exe = _build(tmp_path)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert "c-abi ok" in r.stdout
