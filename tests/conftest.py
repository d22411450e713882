import os
import sys

import pytest

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (sm_100) and the built libgfxb200.so")


@pytest.fixture(scope="session")
def oracle():
    from oracle_lib import Oracle

    return Oracle()
