"""CPU checks of the unit-major plug stream format (no GPU).

The numpy writer and the independent reader in ``unit_plugs_ref`` must round
trip every plug set; the library's size bound (a host-only call) must cover
every stream; and the per-row correction read from the stream must equal the
CSR sparse product of the plug table, which is what the separate correction
kernel computes.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import unit_plugs_ref as upr

SHAPES = [(8, 64), (13, 100), (64, 1024), (300, 68), (9, 4), (40, 4096)]


def plug_set(rng, N, K, density, cluster=False):
    return upr.random_plugs(rng, N, K, density, cluster)


@pytest.mark.parametrize("N,K", SHAPES)
@pytest.mark.parametrize("density,cluster", [(0.0, False), (0.05, False), (0.3, True)])
def test_round_trip(N, K, density, cluster):
    rng = np.random.default_rng(N * 131 + K)
    loc, vals = plug_set(rng, N, K, density, cluster)
    stream, off = upr.build(loc, vals, N, K)
    assert off[0] == 0 and off[-1] == stream.size and (np.diff(off.astype(np.int64)) % 16 == 0).all()
    loc2, vals2 = upr.parse(stream, off, N, K)
    # stream order: unit-major, then row, then column -- the same set
    o = np.argsort(loc2, kind="stable")
    assert np.array_equal(loc2[o], loc)
    assert np.array_equal(vals2[o].view(np.uint16), vals.view(np.uint16))


@pytest.mark.parametrize("N,K", SHAPES)
def test_correction_equals_csr(N, K):
    rng = np.random.default_rng(7 + N + K)
    loc, vals = plug_set(rng, N, K, 0.05, cluster=True)
    x = rng.normal(0, 1, size=K).astype(np.float16)
    stream, off = upr.build(loc, vals, N, K)
    got = upr.correction(stream, off, N, K, x)
    ref = np.zeros((4, N))
    for i, p in enumerate(loc):
        ref[:, p // K] += vals[i].astype(np.float64) * float(x[p % K])
    np.testing.assert_allclose(got, ref, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("N,K,P", [(8, 64, 0), (8, 64, 512), (13, 100, 50), (4096, 11008, 2_254_438)])
def test_size_bound_covers_worst_case(N, K, P):
    from polar_pack_b200 import _lib
    lib = _lib.load()
    nbytes, noff = _lib._size_t(), ctypes.c_int64()
    _lib.check(lib.pp_quad_unit_plugs_bytes(N, K, P, ctypes.byref(nbytes), ctypes.byref(noff)))
    T, W, U = upr.shape_units(N, K)
    assert noff.value == U + 1
    # worst case: every unit's count leaves 15 bytes of padding
    worst = U * 32 + 9 * P + 15 * U
    assert nbytes.value >= worst and nbytes.value % 256 == 0
