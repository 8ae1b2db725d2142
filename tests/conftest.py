import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (runs the CUDA path)")


@pytest.fixture(scope="session")
def gpu_available():
    from ad_b200 import runtime as rt
    return rt.device_count() > 0
