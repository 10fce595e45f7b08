"""Test configuration: the `gpu` marker and shared helpers.

Tests marked ``gpu`` need a B200 (sm_100) and the in-tree libb200q.so; they
are deselected on CPU-only machines with ``-m "not gpu"`` and skipped when no
CUDA device is visible.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden" / "reference_ops.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU and the in-tree CUDA library")


def _cuda_available() -> bool:
    try:
        import torch

        return bool(torch.cuda.is_available())
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN)


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle as O

    O.lib()
    return O
