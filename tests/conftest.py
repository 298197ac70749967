"""Shared test set-up.

Markers: `gpu` tests need a CUDA device (a B200); everything else runs on the
CPU.  The oracle (oracle/dip_oracle.py) is imported only here in tests, as the
checker.
"""
import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
PKG_DIR = REPO / "dynamic-input-pruning_b200"
for p in (str(REPO), str(PKG_DIR)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a)")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def dev():
    import torch
    return torch.device("cuda", 0)


@pytest.fixture(scope="session")
def dip():
    import dip_b200  # loads the sm_100a libraries; raises if they are missing
    return dip_b200


@pytest.fixture(scope="session")
def oracle():
    from oracle import dip_oracle
    return dip_oracle
