import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device and the built library")


@pytest.fixture(scope="session")
def golden():
    """The reference-generated fixtures, grouped by case name."""
    import numpy as np

    z = np.load(os.path.join(ROOT, "tests", "golden", "reference_kda.npz"))
    out = {}
    for key in z.files:
        case, name = key.split("/", 1)
        out.setdefault(case, {})[name] = z[key]
    return out
