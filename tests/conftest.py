"""pytest configuration: the `gpu` marker and import paths.

Tests marked `gpu` need a B200 (they call libct_b200.so through its C ABI);
everything else runs on the CPU: the oracle against the reference's golden
vectors, the ABI layout / export checks and the host-side dispatcher logic.
"""
import importlib
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (REPO, os.path.join(REPO, "oracle"), os.path.join(REPO, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) and libct_b200.so")


@pytest.fixture(scope="session")
def ctb():
    return importlib.import_module("cohere-transcribe_b200")


@pytest.fixture(scope="session")
def wmod():
    return importlib.import_module("cohere-transcribe_b200.weights")
