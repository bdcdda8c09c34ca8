import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "nemotron-super-8gb_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a)")
    config.addinivalue_line("markers", "slow: longer CPU test")


@pytest.fixture(scope="session")
def golden():
    import json

    import numpy as np
    d = os.path.join(ROOT, "tests", "golden")
    g = dict(np.load(os.path.join(d, "golden.npz")))
    with open(os.path.join(d, "golden.json")) as f:
        g["meta"] = json.load(f)
    return g
