import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) and libtrmoe.so")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reflib():
    from oracle.oracle import RefLib
    if not RefLib.available():
        pytest.skip("oracle/_ref (the reference compiled from its sources) is not built here")
    return RefLib()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a GPU")
    from trochilus_b200 import moe
    moe.lib()  # raises when libtrmoe.so is missing: no fallback
    return torch
