"""Shared fixtures. GPU tests are marked ``gpu``; everything else runs on a CPU-only box."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA library)")
    config.addinivalue_line("markers", "slow: full-size cases (seconds of CPU oracle work)")


@pytest.fixture(scope="session")
def pkg():
    import __graft_entry__
    return __graft_entry__.load_package()


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle
    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def engine(pkg):
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    e = pkg.Engine(0)
    yield e
    e.close()
