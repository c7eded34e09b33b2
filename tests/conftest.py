"""Shared fixtures.  Tests marked ``gpu`` need a B200 (sm_100) and the built
CUDA library; everything else runs on the CPU."""
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA library")
    config.addinivalue_line("markers", "slow: larger CPU test")


@pytest.fixture(scope="session")
def golden():
    def load(name):
        with np.load(GOLDEN / name) as f:
            return {k: f[k] for k in f.files}
    return load


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test run without a CUDA device")
    from metallora_b200 import kernels
    if not kernels.is_metal_available():
        pytest.fail("CUDA extension not loadable or device is not sm_100")
    return torch.device("cuda:0")


def rel_err(a, b):
    """Normwise relative error ||a-b|| / ||b||."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
