"""pytest configuration: the `gpu` marker (tests that need a B200; run with -m gpu), the repository root on sys.path,
and session fixtures for the built library and the oracle."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (a B200); run with -m gpu")


@pytest.fixture(scope="session")
def tmlib():
    """libtm_b200.so, built for sm_100a if it is missing or stale (nvcc cross-compiles without a GPU)."""
    from tallymap_b200 import _lib
    _lib.build()
    return _lib


@pytest.fixture(scope="session")
def orc():
    """the CPU oracle (test infrastructure), built for this host's CPU."""
    from oracle import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
