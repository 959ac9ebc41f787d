import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


@pytest.fixture(scope="session", autouse=True)
def _built():
    """Build the oracle (and the library when its sources changed) once per session."""
    from oracle.build import build_oracle
    build_oracle()
    lib = os.path.join(ROOT, "nebula_b200", "libhq.so")
    if not os.path.exists(lib):
        from nebula_b200.build import build
        build()
    yield
