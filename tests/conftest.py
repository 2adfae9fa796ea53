import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "qmesh-afd-tp3_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA sm_100 device (B200)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def cuda_ready():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test collected without a CUDA device")
    from qmesh_b200 import build
    build.build()
    return torch.device("cuda:0")


GOLDEN = ROOT / "tests" / "golden"
