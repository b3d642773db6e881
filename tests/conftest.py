"""Test setup: the `gpu` marker, import paths and shared fixtures.

`-m "not gpu"` runs on a CPU-only machine: the oracle against the golden
vectors, host logic, and the C-ABI library's load/export surface.  `-m gpu`
runs the parity tests of the CUDA path against the oracle on a B200.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_PY = os.path.join(ROOT, "hace-fem-hacedle_b200", "python")
for p in (ROOT, PKG_PY):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libhacedle_cuda.so")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


@pytest.fixture(scope="session")
def ctx():
    import torch
    import hacedle_cuda as hc

    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    c = hc.Context(0)
    yield c
    torch.cuda.synchronize()
    c.close()
