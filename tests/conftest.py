import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mojo-gemma4-cpu_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    # test files whose names start with test_zz_ run last
    items.sort(key=lambda it: 1 if os.path.basename(str(it.fspath)).startswith("test_zz_") else 0)


@pytest.fixture(scope="session")
def has_gpu():
    import torch
    return torch.cuda.is_available()
