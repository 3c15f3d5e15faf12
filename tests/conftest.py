"""Shared test setup: the ``gpu`` marker and helpers for seeded payloads."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); parity through the C ABI")


@pytest.fixture(scope="session")
def golden_decoders():
    return np.load(GOLDEN / "decoders.npz")


@pytest.fixture(scope="session")
def golden_encoders():
    return np.load(GOLDEN / "encoders.npz")


@pytest.fixture(scope="session")
def cuda_device():
    """The CUDA device for -m gpu tests; fails (never skips) when absent."""
    import torch

    from pyrite_b200 import _lib

    if _lib.load() is None:
        pytest.fail("libpyrite_b200.so is not built")
    if not torch.cuda.is_available() or _lib.device_count() == 0:
        pytest.fail("gpu-marked test run without a CUDA device")
    return torch.device("cuda:0")
