import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def rnet():
    """The product binding (librnet_b200.so through the C ABI)."""
    return importlib.import_module("resonance-net_b200")


@pytest.fixture(scope="session")
def rdata():
    return importlib.import_module("resonance-net_b200.data")


@pytest.fixture(scope="session")
def orc():
    """The CPU oracle (test infrastructure)."""
    import oracle
    if not os.path.exists(oracle.LIB_ORACLE):
        oracle.build()
    return oracle


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()
    return torch
