import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; run with -m gpu")


@pytest.fixture(scope="session")
def b2p():
    """The loaded C library, initialised on cuda:0 (GPU tests only)."""
    import torch
    from autoane_b200 import _lib
    assert torch.cuda.is_available(), "GPU test run without a visible CUDA device"
    torch.cuda.init()
    lib = _lib.load()
    _lib.call("b2p_init", 0)
    return lib
