"""Shared fixtures.  GPU tests are marked ``gpu``; everything else runs on CPU."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle

    return Oracle()


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN / "golden_vectors.npz"))


@pytest.fixture(scope="session")
def cuda():
    """The C-ABI library, initialised on device 0 (GPU tests only)."""
    import torch

    from freemoe_b200 import hotpath

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    hotpath.init(0)
    torch.cuda.init()
    return hotpath
