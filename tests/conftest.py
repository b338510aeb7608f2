"""pytest configuration: the ``gpu`` marker selects tests that need a B200."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    return np.load(REPO / "tests" / "golden" / "reference_golden.npz")


@pytest.fixture(scope="session")
def cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from maple_flash_dgx_spark_b200 import _lib

    _lib.lib()  # fail loudly if the library is missing on a GPU box
    return torch.device("cuda", 0)
