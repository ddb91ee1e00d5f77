import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; runs the CUDA path through the C ABI")


def pytest_collection_modifyitems(config, items):
    # GPU tests fail loudly (no skip) when CUDA is missing, except when the run
    # explicitly deselects them with -m "not gpu".
    pass


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from toy_b200 import _lib
    _lib.lib()
    return torch.device("cuda:0")
