import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device and the built extension")
    config.addinivalue_line("markers", "slow: long-running CPU test")
    config.addinivalue_line("markers", "dist: multi-process test (gloo on CPU)")


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(0)
    yield


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
