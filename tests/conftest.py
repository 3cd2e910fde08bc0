import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libjsx.so")
    config.addinivalue_line("markers", "slow: long-running (full-size shapes)")


def pytest_collection_modifyitems(config, items):
    # keep the no-allocation entry point's test last even under -k selections
    items.sort(key=lambda it: os.path.basename(str(it.fspath)).startswith("test_zz"))


@pytest.fixture(scope="session")
def jsx():
    return importlib.import_module("e2e-jaxscale_b200")


@pytest.fixture(scope="session")
def ref():
    return importlib.import_module("oracle.glm4_ref")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", torch.cuda.current_device())
