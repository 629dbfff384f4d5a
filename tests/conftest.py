"""Shared pytest configuration.

`-m gpu` tests need a B200 and the compiled library; `-m "not gpu"` tests run
on any host (oracle, host logic, C ABI load/exports, argument contracts).
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100) device and libthunderfft_b200.so")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import thunderfft_b200 as tf

    tf.load_library()  # raises if the native library is missing: no fallback
    return torch.device("cuda", 0)
