"""Shared fixtures. Tests marked `gpu` need a B200 and run libqms_cuda through its C ABI;
everything else runs on CPU (oracle vs golden vectors, host logic, library symbols)."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests" / "golden"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA sm_100 device (B200)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle import Reference, reference_available
    if not reference_available():
        pytest.skip("oracle/_ref (the reference built from its sources) is not present")
    r = Reference()
    return r


@pytest.fixture(scope="session")
def golden():
    return np.load(ROOT / "tests" / "golden" / "reference_golden.npz")


@pytest.fixture(scope="session")
def cuda():
    """torch + libqms_cuda on cuda:0; fails (not skips) when the CUDA library is missing."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import large_model_b200 as q
    q.init(0)
    torch.cuda.set_device(0)
    return q


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
