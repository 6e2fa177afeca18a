import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; run with -m gpu")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O  # oracle/oracle.py, builds its library on first use

    O.lib()
    return O


@pytest.fixture(scope="session")
def native():
    from purebee_b200 import build

    build.build()
    from purebee_b200 import _native

    _native.lib()
    return _native


@pytest.fixture(scope="session")
def ctx(native):
    c = native.Context(0)
    yield c
    c.close()
