"""Test configuration: the ``gpu`` marker and shared fixtures.

``-m "not gpu"`` runs here without a GPU: the oracle against the golden
fixtures and the reference's host code, and the C-ABI library's exports.
``-m gpu`` runs the parity tests proper on a B200, through the C ABI.
"""
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a) and the compiled library")


def golden(name):
    p = GOLDEN / name
    if not p.exists():
        pytest.skip(f"golden fixture {name} not generated yet (tests/golden/make_golden.py)")
    return np.load(p)


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but CUDA is unavailable")
    return torch.device("cuda:0")
