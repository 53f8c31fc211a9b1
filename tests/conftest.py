"""Shared pytest setup: import paths, the `gpu` marker, golden fixtures."""
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TESTS = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.join(REPO, "vllm-ascend910_b200")
for p in (REPO, PKG_ROOT, TESTS):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def golden():
    return np.load(os.path.join(REPO, "tests", "golden", "golden.npz"))


@pytest.fixture(scope="session")
def orc():
    import oracle
    try:
        oracle.lib()
    except FileNotFoundError:
        import subprocess
        subprocess.check_call(["make", "-s", "-C", os.path.join(REPO, "oracle")])
    return oracle
