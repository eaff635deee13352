"""pytest configuration: the ``gpu`` marker, import paths and native builds.

``-m "not gpu"`` runs on any machine; ``-m gpu`` needs a B200.  The native
library and the CPU oracle are (re)built here when their sources changed.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_ROOT = ROOT / "fast-compressai_b200"
for p in (str(ROOT), str(PKG_ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")
    config.addinivalue_line("markers", "slow: long-running case")
    import build_native  # noqa: E402  (fast-compressai_b200/build_native.py)

    from oracle import oracle as _oracle

    if os.environ.get("FCAI_SKIP_BUILD") != "1":
        build_native.build()
        _oracle.build()


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("a CUDA device is required for -m gpu tests")
    return torch.device("cuda:0")
