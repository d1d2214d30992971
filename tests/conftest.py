"""pytest configuration: the `gpu` marker and shared fixtures.

`-m "not gpu"` runs on any machine (oracle vs golden vectors, host logic, the
C ABI's exported symbols, multi-rank host logic over gloo).  `-m gpu` runs the
parity tests of the CUDA kernels against the oracle; they need a B200.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a) and the built libfd_b200.so")


@pytest.fixture(scope="session")
def golden():
    from tests._golden import load_golden

    return load_golden()
