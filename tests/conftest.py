import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle
    oracle.lib()
    return oracle


@pytest.fixture(autouse=True)
def cr_arithmetic_by_default():
    """Tests compare against the CPU oracle, which restates the correctly
    rounded model; a test of the reference-GPU arithmetic selects "gpu" itself."""
    from concord_b200 import packed_b
    packed_b.set_arithmetic("cr")
    yield
    packed_b.set_arithmetic("gpu")
