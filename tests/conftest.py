"""Shared pytest configuration: the `gpu` marker and common fixtures.

Tests marked ``gpu`` need a B200 (sm_100a) and the built CUDA library; everything else runs
on the CPU (oracle checks, host tiling math, C-ABI symbol checks, gloo multi-process logic).
"""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA library")


@pytest.fixture(scope="session")
def root() -> Path:
    return ROOT


@pytest.fixture(scope="session")
def cuda_torch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch
