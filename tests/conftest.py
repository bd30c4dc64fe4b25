"""Shared test set-up: import paths, the `gpu` marker and common helpers."""

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(REPO, "flash-attention-cuda_b200")
ORACLE_DIR = os.path.join(REPO, "oracle")
for p in (PKG_DIR, ORACLE_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line(
        "markers", "gpu: needs a B200 (sm_100a) GPU; run with -m gpu")


def cuda_available():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


requires_gpu = pytest.mark.skipif(not cuda_available(),
                                  reason="CUDA device required")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(os.path.join(REPO, "tests", "golden", "golden.npz"))
