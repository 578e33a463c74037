"""Shared fixtures.  GPU tests are marked `gpu`; everything else runs on CPU.

The session builds libpackr_b200.so and the oracle's C library in-tree if they
are missing (nvcc/gcc only, no GPU needed)."""
import sys
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def pytest_sessionstart(session):
    from packr_b200 import build as pbuild
    from oracle import build as obuild
    pbuild.build()
    obuild.build_oracle()


@pytest.fixture(scope="session")
def device():
    if torch.cuda.is_available():
        return torch.device("cuda")
    return torch.device("cpu")


@pytest.fixture(scope="session")
def cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    return torch.device("cuda")
