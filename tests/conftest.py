"""Shared fixtures.  `-m gpu` tests need a B200; everything else runs on CPU."""
import importlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (runs the CUDA path through the C ABI)")


@pytest.fixture(scope="session")
def vx():
    return importlib.import_module("webgpu-voxtral_b200")


@pytest.fixture(scope="session")
def synth():
    return importlib.import_module("webgpu-voxtral_b200.synth")


@pytest.fixture(scope="session")
def golden():
    return np.load(os.path.join(ROOT, "tests", "golden", "c1_small.npz"))


def max_abs_rel(a, b) -> float:
    """Parity metric: max|a - b| / max|b| per tensor (tolerance 2e-2 for the f16 path)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))
