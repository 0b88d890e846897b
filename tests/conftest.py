import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(REPO, "tests", "golden")
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: long-running CPU oracle case")


def golden(name):
    path = os.path.join(GOLDEN, name)
    if name.endswith(".npz"):
        return np.load(path)
    return path


@pytest.fixture(scope="session")
def ptlib():
    """The product library; GPU tests fail loudly if it is missing."""
    import pitorch_b200
    return pitorch_b200.lib()


def rel_err(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))
