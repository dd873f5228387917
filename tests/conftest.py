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


@pytest.fixture(scope="session")
def quadpack_small_stream(quadpack_golden):
    """The complete reference-written ``.quadpack`` of ``quadpack_small.npz``.

    The fixture file keeps only the header, two code windows and the tails;
    the oracle writer rebuilds the whole stream from the recorded seed, and
    its SHA-256 must equal the one recorded from the reference's own
    ``pack_quad`` -- so the bytes returned are the reference's bytes.
    """
    import hashlib

    from make_golden import correlated_models
    from oracle import formats as of
    g = quadpack_golden
    seed, n, *extra = (int(x) for x in g["seed_models"])
    flat = correlated_models(np.random.default_rng(seed), 4, (n + max(extra),))
    models = [flat[k][: n + extra[k]].astype(np.float32) for k in range(4)]
    buf = of.pack_quad_bytes(models)
    assert hashlib.sha256(buf).hexdigest() == str(g["sha256"])
    return buf
