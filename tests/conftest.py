"""Shared pytest configuration.

``-m "not gpu"`` runs on a CPU-only machine (oracle vs golden fixtures, host logic, the C-ABI
library's exported symbols and struct layouts, gloo multi-rank exchange logic).  ``-m gpu`` are
the parity tests proper: the CUDA kernels, called through the C ABI, against the CPU oracle."""

import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (run on the B200 box)")


@pytest.fixture(scope="session")
def norm_golden():
    return torch.load(GOLDEN / "norm_golden.pt", weights_only=True)


@pytest.fixture(scope="session")
def softmax_ce_golden():
    return torch.load(GOLDEN / "softmax_ce_golden.pt", weights_only=True)


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(0)
    yield


@pytest.fixture(scope="session")
def linear_ce_golden():
    return torch.load(GOLDEN / "linear_ce_golden.pt", weights_only=True)
