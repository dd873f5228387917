"""Shared pytest set-up: the ``gpu`` marker, repo import paths, fixture loaders."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
for p in (str(ROOT), str(GOLDEN)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200 / sm_100a)")


def golden(name: str):
    return np.load(GOLDEN / f"{name}.npz")


@pytest.fixture(scope="session")
def quad_golden():
    return golden("quad_layer")


@pytest.fixture(scope="session")
def dual_golden():
    return golden("dual_layer")


@pytest.fixture(scope="session")
def quadpack_golden():
    return golden("quadpack_small")


@pytest.fixture(scope="session")
def dualpack_golden():
    return golden("dualpack_small")


def bits(x) -> np.ndarray:
    """FP16 array as its uint16 bit patterns (exact comparison incl. -0)."""
    return np.asarray(x, dtype=np.float16).view(np.uint16)


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from polar_pack_b200 import _lib
    _lib.load()
    return torch.device("cuda", 0)
