import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs on a B200)")
    config.addinivalue_line("markers", "slow: full-size model parity (minutes of oracle CPU time)")


@pytest.fixture(scope="session")
def device():
    """Initialises the CUDA device through the C ABI (GPU tests only)."""
    from brewference_b200 import _native as N
    N.init(0)
    return 0
