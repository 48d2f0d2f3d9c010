"""pytest configuration: the ``gpu`` marker and import paths.

Tests marked ``gpu`` need a B200 and the built ``libtfb200.so``; everything else
runs on a CPU-only machine.
"""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "tt-flow_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device and the built CUDA library")


@pytest.fixture(scope="session")
def golden_vectors():
    import numpy as np

    return np.load(ROOT / "tests" / "golden" / "golden_vectors.npz")
