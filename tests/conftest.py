import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(Path(__file__).resolve().parent))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def _cuda_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def cuda_device():
    """The GPU tests run only where a CUDA device exists; they fail (not skip) when the library is missing."""
    if not _cuda_available():
        pytest.skip("no CUDA device in this environment")
    from ripvec_b200 import _lib

    _lib.lib()  # raises if librv_b200.so was not built
    return int(os.environ.get("RV_TEST_DEVICE", "0"))
