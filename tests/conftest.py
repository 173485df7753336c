import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "multigpu: needs two or more GPUs")


@pytest.fixture(scope="session")
def cuda_lib():
    """The CUDA library; on a GPU run its absence is an error, never a skip."""
    import torch
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    from tinylama_b200 import _lib
    return _lib
