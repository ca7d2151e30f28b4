"""Shared pytest configuration.

Tests marked ``gpu`` need a CUDA device (a B200); everything else runs on a
CPU-only host.  The oracle (oracle/) is built on demand for the CPU tests.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(os.path.join(ROOT, "tests", "golden", "golden.npz"))


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle as O
    O.port()
    return O
