import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
TESTS = os.path.dirname(os.path.abspath(__file__))
if TESTS not in sys.path:
    sys.path.insert(0, TESTS)


def pytest_addoption(parser):
    parser.addoption("--crosslane-ref", default=None,
                     help="crosslane checkout for the tests that compile against its headers")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (run with -m gpu on a B200)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def orc():
    import oracle_lib
    return oracle_lib.Oracle()


@pytest.fixture(scope="session")
def ref():
    import oracle_lib
    r = oracle_lib.reference()
    if r is None:
        pytest.skip("oracle/_ref/libref.so (crosslane's own arithmetic) not built on this machine")
    return r


@pytest.fixture(scope="session")
def scale_table(orc):
    return orc.scale_table()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch
