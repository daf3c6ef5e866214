"""Shared test setup: import paths, the gpu marker, common fixtures."""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "zonos2.cpp_b200")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def oracle():
    from oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for gpu-marked tests")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def z2():
    import zonos2cu
    zonos2cu.lib()  # fails loudly when the library is missing
    return zonos2cu
