"""Shared fixtures.  GPU tests carry @pytest.mark.gpu and run on a B200 box; every
other test runs on a CPU-only machine."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: full-size case (minutes of CPU oracle work)")


@pytest.fixture(scope="session")
def oracle():
    import oracle as orc
    orc.build()
    return orc


@pytest.fixture(scope="session")
def ctx():
    """One library context on cuda:0 for the whole GPU session."""
    import pion_b200
    c = pion_b200.Context(0)
    yield c
    c.close()


@pytest.fixture
def rng():
    return np.random.Generator(np.random.PCG64(1974))
