import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library")


def golden(name):
    """A committed fixture made by tests/golden/make_golden.py from the reference."""
    return np.load(os.path.join(GOLDEN, name))


@pytest.fixture
def gold():
    return golden
