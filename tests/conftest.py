import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built gpb200 library")


@pytest.fixture(scope="session")
def gpb_lib():
    """The built CUDA library (built on demand; never a CPU fallback)."""
    from mojogp_b200 import build
    build.build()
    from mojogp_b200 import _lib
    return _lib.lib()


def rel_fro(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))
