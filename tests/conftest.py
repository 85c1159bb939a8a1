"""Shared test fixtures. Tests marked `gpu` need a B200 and run through the C ABI; all other
tests run on the CPU (the oracle against golden vectors, host logic, library exports)."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU (sm_100a); runs through the C ABI")


@pytest.fixture(scope="session")
def built_lib():
    """The in-tree C-ABI library, built if missing (nvcc cross-compiles without a GPU)."""
    from transfer_station_b200 import build

    build.build()
    import transfer_station_b200 as ts

    return ts.load_library()


@pytest.fixture(scope="session")
def cuda_dev(built_lib):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, _ = torch.cuda.get_device_capability(0)
    assert major == 10, "the GPU tests need a compute capability 10.x (B200) device"
    return torch.device("cuda:0")
