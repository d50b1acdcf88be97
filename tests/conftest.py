import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built libenvgemm.so")


@pytest.fixture(scope="session")
def gpu():
    """Initialise libenvgemm on cuda:0 once per session (GPU tests only)."""
    from invision_b200 import envg

    envg.init(0)
    return envg
