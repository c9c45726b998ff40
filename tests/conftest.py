import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "enigma-dsl_b200"))
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available() and torch.cuda.get_device_capability(0)[0] == 10
    except Exception:
        return False


@pytest.fixture(scope="session")
def cuda():
    if not has_gpu():
        pytest.fail("this test needs a B200 GPU (run with -m 'not gpu' on CPU hosts)")
    import torch
    return torch.device("cuda:0")
