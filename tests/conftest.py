import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device and the built library")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    def load(name):
        return np.load(ROOT / "tests" / "golden" / f"{name}.npz")
    return load
