import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "psp-ml_b200"))
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def ctx():
    """One pspml context on cuda:0 for the GPU tests."""
    import torch
    from pspml import capi

    assert torch.cuda.is_available(), "GPU test needs a CUDA device"
    torch.cuda.init()
    c = capi.Context(0)
    c.set_timeout_ms(60_000)
    yield c
    c.close()


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle as orc
    orc.lib()
    return orc
