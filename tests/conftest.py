"""Shared pytest configuration.

Tests marked ``gpu`` need a CUDA device (a B200 for the sm_100a library) and
call the kernels through the C ABI.  They fail, rather than skip, when no GPU
is present, so a GPU run can never pass on a silent fallback.  Everything else
runs on the CPU.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device and the built sm_100a library")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device; run it on the GPU box (pytest -m gpu)")
    return torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _seed():
    import torch

    torch.manual_seed(0)
    os.environ.setdefault("PYTHONHASHSEED", "0")
    yield
