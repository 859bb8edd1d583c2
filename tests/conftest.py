"""Test configuration: the `gpu` marker and shared fixtures.

`-m "not gpu"` runs on any host (oracle pins, host logic, C-ABI loading and
validation); `-m gpu` runs the CUDA parity tests and needs a B200.
"""
import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built library")


@pytest.fixture(scope="session")
def spt():
    return importlib.import_module("stream-pt_b200")


@pytest.fixture(scope="session")
def ctx(spt):
    c = spt.Context(0)
    yield c
    c.close()


@pytest.fixture(scope="session")
def host_ctx(spt):
    c = spt.Context(-1)
    yield c
    c.close()
