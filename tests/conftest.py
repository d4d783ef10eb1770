"""pytest configuration: the `gpu` marker and shared fixtures."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200 / sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs 2 or more CUDA GPUs")


@pytest.fixture(scope="session")
def ext():
    """The native extension; on a GPU run a missing build is a failure, not a skip."""
    from ring_attention_benchmark_b200 import _ext

    return _ext.load()


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but torch.cuda.is_available() is False")
    return torch.device("cuda", 0)
