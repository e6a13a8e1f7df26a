"""Test configuration: the `gpu` marker, import paths and shared fixtures.

-m "not gpu" runs on any machine (oracle pins, C-ABI symbol checks, host
logic, gloo multi-process logic); -m gpu needs a CUDA device and calls the
kernels through the C ABI.
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT / "oracle", ROOT / "whisper-xdna_b200", ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long CPU oracle (large-v3 depth)")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test run without a CUDA device")
    return torch.device("cuda", 0)


@pytest.fixture(scope="session")
def wxlib():
    from wxb200 import _lib
    return _lib.lib()
