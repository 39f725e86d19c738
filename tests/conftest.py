"""Shared test setup: import paths, the `gpu` marker, seeded inputs, metrics."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "attn-cpu_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
GOLDEN = os.path.join(ROOT, "tests", "golden", "reference_vectors.npz")

# Parity bars (max|y - r| / max|r| against the oracle / the reference).
TOL_3XTF32 = 1e-5
TOL_TF32 = 2e-3
TOL_FP32 = 1e-5  # CUDA-core fp32 paths (decode, generic prefill)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) CUDA device")


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN)


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    return torch.device("cuda:0")


def rel_err(y, r) -> float:
    y = np.asarray(y, np.float64)
    r = np.asarray(r, np.float64)
    if r.size == 0:
        return 0.0
    den = float(np.max(np.abs(r)))
    num = float(np.max(np.abs(y - r)))
    return num / den if den > 0 else num
