"""pytest configuration: the `gpu` marker and import paths.

Tests marked `gpu` need a CUDA device (a B200) and call the product through its
C-ABI; everything else runs on CPU.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mobile-moe.zig_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); runs the product kernels")


@pytest.fixture(scope="session")
def oracle():
    import kvoracle

    kvoracle.build()
    return kvoracle


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    return np.load(os.path.join(ROOT, "tests", "golden", "golden.npz"))
