import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: long-running parity case")


@pytest.fixture(scope="session")
def oracle():
    import oracle as o
    o.build()
    return o


@pytest.fixture(scope="session")
def faber():
    from faber_runtime_b200 import build
    build.build()
    import faber_runtime_b200 as fb
    fb.lib()
    return fb


@pytest.fixture(scope="session")
def cuda(faber):
    """The CUDA device for -m gpu tests (fails loudly without one)."""
    import torch
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    from faber_runtime_b200 import _lib
    _lib.call("faber_gpu_v2_init", 0)
    return torch.device("cuda:0")
