"""Shared pytest setup: import paths, the ``gpu`` marker, device fixtures.

``-m "not gpu"`` runs on any machine (oracle vs golden vectors, host logic,
the C ABI's exported symbols, gloo multi-rank tests); ``-m gpu`` needs a B200
and calls the kernels through the C ABI.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "bitsandbytes-jax_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a)")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(ROOT / "tests" / "golden" / "reference_golden.npz")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.skip(f"needs sm_100 (B200), found sm_{major}{minor}")
    return torch.device("cuda:0")


@pytest.fixture(scope="module")
def timeouts_at_start(cuda):
    """The device's count of expired bounded waits when the module starts
    (the count is process-wide; a test that makes waits expire on purpose
    raises it for every later module)."""
    import torch
    from bnb_b200 import _lib
    torch.cuda.synchronize()
    return _lib.wait_timeouts()
