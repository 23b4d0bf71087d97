"""Shared test setup: the `gpu` marker, import paths, and helpers.

`-m "not gpu"` tests run on the CPU: the oracle against the reference's own
golden vectors and thresholds, host logic, and that the C-ABI library loads
and exports every declared symbol. `-m gpu` tests run the CUDA path through
the C ABI and compare it with the oracle.
"""
import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE = os.path.join(ROOT, "oracle")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, ORACLE):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def lumen():
    """The product package (directory name lumen-rs_b200)."""
    return importlib.import_module("lumen-rs_b200")


def have_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def lc():
    return lumen()


@pytest.fixture(scope="session")
def orc():
    import pyoracle

    pyoracle.build()
    return pyoracle


@pytest.fixture(scope="session")
def gpu():
    if not have_gpu():
        pytest.fail("this test needs a CUDA GPU")
    return 0
