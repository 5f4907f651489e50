"""Shared pytest configuration.  Tests marked ``gpu`` need a CUDA device and the built
``libopc_b200.so``; everything else runs on CPU."""

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and libopc_b200.so")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    # The library must be present on a GPU machine: failing to load it is an error, not a skip.
    from opac1ty_b200 import _lib

    _lib.load()
    return torch.device("cuda", 0)
