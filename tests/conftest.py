"""Shared pytest setup.

Markers: ``gpu`` — needs a CUDA device (run with ``-m gpu`` on a B200).
Without a GPU the suite covers the oracle against the golden vectors, the
host-side logic and that libhxkv.so loads and exports its ABI.
"""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def _ensure_oracle():
    lib = os.path.join(ROOT, "oracle", "liboracle.so")
    src = os.path.join(ROOT, "oracle", "hx_oracle.c")
    if not os.path.exists(lib) or os.path.getmtime(src) > os.path.getmtime(lib):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "all"], check=True)


_ensure_oracle()


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    return O


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(os.path.join(ROOT, "tests", "golden", "reference_golden.npz"))


@pytest.fixture(scope="session")
def hxlib():
    from hxinfer_b200 import _lib
    return _lib.load()
