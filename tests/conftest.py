"""Test configuration: `-m gpu` tests need a B200 and the in-tree native libraries;
everything else runs on the CPU (oracle, golden vectors, host logic, ABI exports)."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "system1-omni_b200"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built libraries")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(scope="session")
def cs1():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from s1omni import Cs1
    lib = Cs1()
    torch.cuda.init()
    return lib


@pytest.fixture
def stream():
    import torch
    return torch.cuda.current_stream().cuda_stream
