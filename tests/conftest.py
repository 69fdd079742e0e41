"""Shared test set-up: the `gpu` marker, the repository on sys.path, and the CPU checkers (oracle/) built on demand."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (a B200)")


@pytest.fixture(scope="session", autouse=True)
def _oracle_built():
    import oracle
    if not os.path.exists(oracle.ORACLE_SO) or (not oracle.ref_available() and os.path.isdir(oracle.REF_DIR_DEFAULT)):
        oracle.build()
    yield


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(os.path.join(ROOT, "tests", "golden", "moe_golden.npz"))
