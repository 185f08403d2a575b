import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

GOLDEN = os.path.join(REPO, "tests", "golden", "golden.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device")


@pytest.fixture(scope="session")
def golden():
    g = np.load(GOLDEN)
    names = sorted({k.split("/")[0] for k in g.files if not k.startswith("meta")})
    return {n: {k.split("/", 1)[1]: g[k] for k in g.files if k.startswith(n + "/")}
            for n in names}
