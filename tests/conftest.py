import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built sm_100a libraries")


def cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as orc
    orc.lib()
    return orc


@pytest.fixture(scope="session")
def gpu():
    """Device + loaded libraries; GPU tests fail (not skip) when the native
    libraries are missing on a GPU box, so a silent fallback cannot pass."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import time_b200
    time_b200.load()
    torch.cuda.set_device(0)
    return torch.device("cuda:0")
