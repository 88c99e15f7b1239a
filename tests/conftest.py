import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line(
        "markers", "gpu: needs a B200 (sm_100a); run with -m gpu")
    config.addinivalue_line(
        "markers", "multigpu: needs two or more B200s")
    config.addinivalue_line("markers", "slow: takes more than a few seconds")


@pytest.fixture(scope="session")
def cuda_lib():
    """The product library on a GPU box; fails loudly when it is missing."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from reef_b200 import _lib
    return _lib.lib()
