"""Shared pytest configuration.

`-m gpu` tests need a B200 (sm_100a) and the built library
bonsai.cpp_b200/lib/libbonsai_cuda.so; `-m "not gpu"` tests run on CPU only.
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "bonsai.cpp_b200"))
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA library")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def gpu():
    """Initialise device 0 through the C ABI.  Fails (does not skip) when no
    GPU is visible: gpu-marked tests only run where one must exist."""
    import torch
    import bonsai_b200 as bb
    assert torch.cuda.is_available(), "gpu-marked test run without a visible CUDA device"
    torch.cuda.init()
    bb.init(0)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield bb
    assert bb.device_error() == 0, "a kernel reported a device-side timeout"
