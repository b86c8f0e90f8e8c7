import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
if str(ROOT / "tests") not in sys.path:
    sys.path.insert(0, str(ROOT / "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100) device")


@pytest.fixture(scope="session")
def dev():
    import torch

    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    torch.cuda.set_device(0)
    return torch.device("cuda:0")


@pytest.fixture()
def blas(dev):
    from grxcp_b200 import blas as B

    h = B.Handle()
    yield h
    h.close()


@pytest.fixture()
def dnn(dev):
    from grxcp_b200 import dnn as D

    h = D.Handle()
    yield h
    h.close()
