import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
TESTS = os.path.dirname(os.path.abspath(__file__))
if TESTS not in sys.path:
    sys.path.insert(0, TESTS)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def g2():
    import g2util

    return g2util.load_pkg()


@pytest.fixture(scope="session")
def oracle():
    import g2util

    return g2util.Oracle()


@pytest.fixture(scope="session")
def ref():
    import g2util

    r = g2util.Reference.load()
    if r is None:
        pytest.skip("oracle/_ref/libggemm_ref.so not built (needs the reference sources)")
    return r


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
