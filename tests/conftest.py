"""Shared pytest setup: the ``gpu`` marker and import paths.

``-m "not gpu"`` runs on a CPU-only host (oracle vs golden vectors, packer,
host-side logic, C-ABI symbol exports, gloo multi-process bookkeeping).
``-m gpu`` runs the parity tests proper through the C-ABI on a B200.
"""
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "triposplat-cpu-avx512_b200"
for p in (str(REPO), str(PKG), str(REPO / "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import Oracle

    return Oracle()


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    def load(name):
        return dict(np.load(GOLDEN / f"{name}.npz"))

    return load
