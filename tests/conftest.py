"""Shared pytest configuration.

Tests marked ``gpu`` need a B200 and the built libenl_b200.so; everything
else runs on the CPU (oracle pins, host logic, ABI symbol checks, gloo
multi-process tests).
"""
import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) GPU and libenl_b200.so")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


@pytest.fixture(scope="session")
def cuda():
    """Skip-free guard: a gpu-marked test on a box without a GPU is an error,
    not a silent pass."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test selected but torch.cuda.is_available() is False")
    from enilnets_b200 import _native
    _native.load()
    return torch.device("cuda", 0)
