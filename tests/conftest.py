import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "qvex-3.5_b200"
for p in (PKG, ROOT / "oracle", ROOT / "tests" / "golden", ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built libqvex.so")
    config.addinivalue_line("markers", "slow: takes more than a few seconds")


def pytest_runtest_setup(item):
    if item.get_closest_marker("gpu") is not None:
        import torch
        if not torch.cuda.is_available():
            pytest.fail("GPU test selected but no CUDA device is visible")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle
    oracle.build()
    return oracle
