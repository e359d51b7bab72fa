"""Shared test set-up: the ``gpu`` marker, fixture loading and GPU gating."""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a) and the built CUDA library")
    config.addinivalue_line("markers", "slow: long running tests")


def golden(name: str):
    """Load ``tests/golden/<name>.npz`` (generated from the reference by make_golden.py)."""
    return np.load(GOLDEN / f"{name}.npz", allow_pickle=False)


@pytest.fixture
def cuda():
    """The CUDA device for ``-m gpu`` tests; skips when no GPU is visible."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    return torch.device("cuda", 0)


def pytest_collection_modifyitems(config, items):
    # GPU tests fail loudly (not skip) when a GPU is present but the library is not
    # built: the product path has no fallback.
    os.environ.setdefault("LINATTN_B200_STRICT", "1")
