"""Test configuration: `gpu` marks tests that need a B200; everything else runs on the CPU."""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and librldx_b200.so")
    config.addinivalue_line("markers", "slow: long-running parity case")


@pytest.fixture(scope="session")
def lib():
    import rldx_b200  # noqa: F401
    from rldx_b200 import _lib

    return _lib.load()


@pytest.fixture(scope="session")
def cuda(lib):
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu test without a CUDA device")
    if lib.rldx_device_supported() != 1:
        pytest.fail("librldx_b200 reports the device as unsupported: " + lib.rldx_last_error().decode())
    return torch.device("cuda", 0)
