"""Test configuration.

Markers: ``gpu`` -- needs a B200 (sm_100a) and the built liblal_tail.so; the
driver runs ``pytest -m gpu`` on a GPU box and ``pytest -m "not gpu"`` on CPU.
The CPU suite covers the oracle against the golden vectors (and against the
reference's own compiled C where oracle/_ref was built), the host logic, the
synthetic-input generators and the C ABI's symbols; the GPU suite is the
parity suite proper and calls through the C ABI.
"""
import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, GOLDEN):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a) and liblal_tail.so")
    config.addinivalue_line("markers", "slow: full-size case (seconds to a minute)")


@pytest.fixture(scope="session")
def golden():
    return np.load(os.path.join(GOLDEN, "golden.npz"))


@pytest.fixture(scope="session")
def golden_meta():
    with open(os.path.join(GOLDEN, "golden.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def port():
    import oracle
    oracle.port()
    return oracle


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.int32)
