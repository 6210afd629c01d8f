"""Shared test setup: the `gpu` marker, the oracle build, and helpers.

Tests marked `gpu` need a CUDA device and call the library through its C ABI;
everything else runs on CPU only (oracle pins, host logic, ABI loading).
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built library")


@pytest.fixture(scope="session")
def oracle():
    import pyoracle

    pyoracle.build()
    return pyoracle


@pytest.fixture(scope="session")
def tb():
    import tendo_b200

    return tendo_b200


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu test without a CUDA device")
    return torch.device("cuda:0")


def rel_err(got, want):
    """max |got - want| / max |want| (the tolerance measure the tests state)."""
    import numpy as np

    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    denom = max(float(np.abs(want).max()), 1e-30)
    return float(np.abs(got - want).max()) / denom
