import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


@pytest.fixture(scope="session")
def native_lib():
    """librumik_b200.so, built in-tree first if it is missing or older than its sources (needs nvcc)."""
    from rumik_fast_b200 import _lib, build
    if not build.up_to_date():
        build.build()
    return _lib.lib()
