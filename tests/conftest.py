"""Shared test set-up: the `gpu` marker, the repository on sys.path, and the CPU checkers (oracle/) built on demand."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


# The reference engine's sources, where this machine has them (the CPU tests that compile against its headers, and the
# on-demand build of oracle/_ref, read them there); a GPU machine without them uses the prebuilt oracle/_ref.
REFERENCE_SRC = "/root/reference/c/src"
if not os.environ.get("CLUTOR_REF_DIR") and os.path.isdir(REFERENCE_SRC):
    os.environ["CLUTOR_REF_DIR"] = REFERENCE_SRC


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (a B200)")


@pytest.fixture(scope="session", autouse=True)
def _oracle_built():
    import oracle
    if not os.path.exists(oracle.ORACLE_SO) or (not oracle.ref_available() and oracle.ref_dir()):
        oracle.build()
    yield


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(os.path.join(ROOT, "tests", "golden", "moe_golden.npz"))
