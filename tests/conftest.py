"""pytest configuration: the `gpu` marker and shared fixtures.

Tests marked ``gpu`` need a B200 (sm_100) and call the CUDA path through the
C ABI; everything else runs on CPU. The oracle package (``oracle/``) is the
checker for both.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200); runs the CUDA path")


def _has_sm100() -> bool:
    try:
        import torch
        return torch.cuda.is_available() and torch.cuda.get_device_capability(0) == (10, 0)
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _has_sm100():
        return
    skip = pytest.mark.skip(reason="needs an sm_100 GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def orc():
    import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def mcb():
    import matcoredsl_b200
    return matcoredsl_b200
