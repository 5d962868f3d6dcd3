import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


def load_samrs():
    """The product package lives in the directory `sam-rs_b200` (not an identifier), so import it by name."""
    return importlib.import_module("sam-rs_b200")


@pytest.fixture(scope="session")
def samrs():
    return load_samrs()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
