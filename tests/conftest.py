import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def golden(name: str):
    return np.load(GOLDEN / name)


@pytest.fixture(scope="session")
def lib_path():
    """The built C-ABI library (built here with nvcc when missing)."""
    from exq_b200 import build as B
    if not B.LIB.exists():
        B.build()
    return B.LIB


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from exq_b200 import build as B
    if not B.LIB.exists():
        B.build()
    torch.cuda.init()
    return torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _seed():
    import torch
    torch.manual_seed(0)
    np.random.seed(0)
    yield
