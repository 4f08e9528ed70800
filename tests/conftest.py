"""Shared pytest configuration: the ``gpu`` marker (tests that need a B200 and the compiled extension) and the
``slow`` marker (multi-process tests)."""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a) and the compiled extension")
    config.addinivalue_line("markers", "slow: spawns processes or runs long")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from economize_b200 import ops

    # CUDA tensors must reach the compiled kernels: a missing extension is a failure, not a skip
    ops.require()
    return torch.device("cuda", 0)
