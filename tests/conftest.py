"""Test configuration: the `gpu` marker and the session build of the native parts."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (runs on the B200 box)")


@pytest.fixture(scope="session", autouse=True)
def native_build():
    """Build the CUDA library, the C++ layer and the oracle once per session (no-op when fresh)."""
    from powersparse_b200 import build
    from oracle import oracle
    build.build_all()
    oracle.build()
    yield
