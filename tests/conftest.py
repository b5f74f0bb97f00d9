import importlib
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libddg.so")


@pytest.fixture(scope="session")
def ddg():
    return importlib.import_module("idash26-track3_b200")


@pytest.fixture(scope="session")
def synth():
    return importlib.import_module("idash26-track3_b200.synth")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    torch.cuda.init()
    return torch
