"""Shared pytest configuration.

``gpu`` marks tests that need a CUDA device (they call the sm_100a library
through its C ABI). Everything else runs on CPU.
"""

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (REPO, os.path.join(REPO, "csaq-quant_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(scope="session")
def kgold():
    import numpy as np
    return np.load(os.path.join(REPO, "tests", "golden", "kernels_golden.npz"))


@pytest.fixture(scope="session")
def cgold():
    import numpy as np
    return np.load(os.path.join(REPO, "tests", "golden", "calib_golden.npz"))


@pytest.fixture(scope="session")
def digests():
    import json
    with open(os.path.join(REPO, "tests", "golden", "digests.json")) as f:
        return json.load(f)
