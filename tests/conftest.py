import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "linalg-gpu-comp_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = ROOT / "tests" / "golden" / "golden_qr.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100) device; run with -m gpu")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(GOLDEN)


def golden_cases():
    import numpy as np
    g = np.load(GOLDEN)
    return [str(c).split(":") for c in g["cases"]]
