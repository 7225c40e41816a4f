import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")
    config.addinivalue_line("markers", "slow: full-size cases")


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(os.path.join(ROOT, "tests", "golden", "golden.npz")))


def golden_group(g, prefix):
    """{case_name: {key: array}} for keys under `prefix/`."""
    out = {}
    for k, v in g.items():
        if k.startswith(prefix + "/"):
            _, case, key = k.split("/", 2)
            out.setdefault(case, {})[key] = v
    return out
