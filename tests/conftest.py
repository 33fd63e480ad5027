import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (a B200); runs the kernels through the C ABI")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    here = os.path.join(REPO, "tests", "golden")
    return {name: np.load(os.path.join(here, name + ".npz")) for name in ("dequant", "route", "moe")}
