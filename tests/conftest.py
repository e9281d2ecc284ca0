import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

import __graft_entry__ as graft  # noqa: E402

graft.load_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libyfattn.so")


@pytest.fixture(scope="session")
def yf():
    return graft.load_package()


@pytest.fixture(scope="session")
def oracle():
    return graft.load_oracle()


@pytest.fixture(scope="session")
def cuda(yf):
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    yf.lib()  # fails loudly if libyfattn.so is missing
    return torch.device("cuda", 0)
