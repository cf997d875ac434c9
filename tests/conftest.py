import sys
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100a (B200) GPU and the built native library")
    config.addinivalue_line("markers", "distributed: spawns torch.distributed gloo process groups")


def has_b200() -> bool:
    return torch.cuda.is_available() and torch.cuda.get_device_capability() == (10, 0)


@pytest.fixture
def cuda():
    if not has_b200():
        pytest.skip("needs an sm_100a GPU")
    from forgeml_b200 import _native

    _native.load()  # a GPU test without the native library is a failure, not a skip
    return torch.device("cuda", 0)
