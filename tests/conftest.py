import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built libfd_b200.so")


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return ROOT / "tests" / "golden"


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    cap = torch.cuda.get_device_capability()
    assert cap[0] == 10, f"expected an sm_100 device, got {cap}"
    return torch.device("cuda:0")


def gen(seed: int):
    import torch

    return torch.Generator().manual_seed(seed)
