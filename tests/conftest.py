import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU (run with -m gpu)")


def load_positions():
    from metalfish_b200.netfile import PackedInputs
    z = np.load(os.path.join(GOLDEN, "positions.npz"))
    return PackedInputs(z["masks"], z["values"])


def load_golden(name):
    z = np.load(os.path.join(GOLDEN, f"ref_{name}.npz"))
    return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def positions():
    return load_positions()
