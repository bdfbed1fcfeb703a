"""Test configuration.

`-m gpu` tests need a CUDA device (they are the parity tests proper and call the
GEMM through libojx's C-ABI); everything else runs on CPU: the oracle against the
reference's golden vectors, the host logic, and the C-ABI library's exports.
"""
import os
import pathlib
import sys

import pytest

REPO = pathlib.Path(__file__).resolve().parents[1]
PKG = REPO / "ojasx-open-source-cuda-_b200"
for p in (str(REPO), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100) device")


def _has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden_dir() -> pathlib.Path:
    return REPO / "tests" / "golden"


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import build_oracle
    build_oracle.build_oracle()
    from oracle import oracle
    return oracle
