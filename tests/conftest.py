"""pytest configuration: the `gpu` marker, import paths, shared fixtures.

`-m "not gpu"` runs the CPU suite (oracle against the golden vectors, host
logic, C-ABI exports, gloo multi-process sharding); `-m gpu` runs the parity
tests through the C ABI on a B200.
"""
import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "cublas-rs_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and libb2blas.so")


def load_golden(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O

    O.build()
    return O


@pytest.fixture(scope="session")
def handle():
    import b2blas

    h = b2blas.Handle(0)
    yield h
    h.close()
