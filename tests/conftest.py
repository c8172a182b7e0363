"""Shared pytest configuration.

Marker ``gpu``: the test needs a CUDA device (B200, sm_100a).  The CPU suite
(`-m "not gpu"`) covers the oracle against the reference's known answers,
the host logic and the C-ABI exports; the `-m gpu` suite holds the parity
tests proper, which call the CUDA path through the C-ABI.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200 / sm_100a)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.lib()
    return O
