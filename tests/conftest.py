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


def pytest_terminal_summary(terminalreporter):
    """The worst max-relative attention error (per (sequence, head) row, against
    the oracle or another kernel path) seen by any test of this session."""
    try:
        import kvdata
    except ImportError:
        return
    if kvdata.WORST["where"]:
        terminalreporter.write_line(f"worst attention error this run: {kvdata.WORST['err']:.3e} "
                                    f"({kvdata.WORST['where']}; tolerance {kvdata.REL_TOL:g})")


@pytest.fixture(scope="session")
def oracle():
    import kvoracle

    kvoracle.build()
    return kvoracle


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    return np.load(os.path.join(ROOT, "tests", "golden", "golden.npz"))
