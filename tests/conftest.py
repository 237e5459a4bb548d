import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (runs on the B200 box)")


@pytest.fixture(scope="session")
def product_lib():
    from compressor_b200 import build as b
    if not os.path.exists(b.OUT):
        b.build()
    return b.OUT


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import binding
    binding.lib()
    return binding
