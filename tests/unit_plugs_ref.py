"""numpy statement of the unit-major plug stream (test helper).

The stream is this library's own load-time layout of a Linear's plug
entries (include/polar_pack_b200.h, pp_quad_prepare_unit_plugs); it has no
reference counterpart.  ``build`` writes it from the plug positions,
``parse`` reads it back independently, and ``correction`` applies it the way
the fused GEMV does (per row, FP64 here).
"""
from __future__ import annotations

import numpy as np


def random_plugs(rng, N: int, K: int, density: float, cluster: bool = False):
    """Sorted positions (density of N*K, plus with ``cluster`` one fully
    plugged 8 x 64 unit) and random FP16x4 values."""
    n = N * K
    loc = rng.choice(n, size=int(n * density), replace=False)
    if cluster and N >= 8 and K >= 64:
        t = rng.integers(0, N // 8)
        kc = rng.integers(0, K // 64)
        blk = ((8 * t + np.arange(8))[:, None] * K + 64 * kc + np.arange(64)).ravel()
        loc = np.union1d(loc, blk)
    loc = np.sort(loc).astype(np.int64)
    vals = rng.normal(0, 1, size=(loc.size, 4)).astype(np.float16)
    return loc, vals


def shape_units(N: int, K: int) -> tuple[int, int, int]:
    W = -(-K // 64)
    T = -(-N // 8)
    return T, W, T * W


def build(loc: np.ndarray, vals: np.ndarray, N: int, K: int) -> tuple[np.ndarray, np.ndarray]:
    """Stream bytes and unit offsets (U + 1, uint32) for ascending positions
    ``loc`` (row * K + column inside the Linear) with FP16x4 ``vals``."""
    loc = np.asarray(loc, dtype=np.int64)
    vals = np.ascontiguousarray(np.asarray(vals, dtype=np.float16).reshape(-1, 4))
    T, W, U = shape_units(N, K)
    row, col = loc // K, loc % K
    unit = (row // 8) * W + col // 64
    counts = np.bincount(unit, minlength=U).astype(np.int64)
    seg = (32 + 9 * counts + 15) // 16 * 16
    off = np.zeros(U + 1, dtype=np.int64)
    off[1:] = np.cumsum(seg)
    out = np.zeros(int(off[-1]), dtype=np.uint8)
    rows = np.bincount(unit * 8 + row % 8, minlength=U * 8).reshape(U, 8)
    end = rows.cumsum(axis=1)
    hdr = ((end - rows) | (end << 10) | (counts[:, None] << 20)).astype("<u4")
    out[off[:U, None] + np.arange(32)] = hdr.view(np.uint8).reshape(U, 32)
    order = np.argsort(unit, kind="stable")  # positions ascend, so rows then columns ascend in a unit
    us = unit[order]
    first = np.zeros(U + 1, dtype=np.int64)
    first[1:] = np.cumsum(counts)
    e = np.arange(loc.size) - first[us]
    out[(off[us] + 32 + 8 * e)[:, None] + np.arange(8)] = vals[order].view(np.uint8).reshape(-1, 8)
    out[off[us] + 32 + 8 * counts[us] + e] = (col[order] % 64).astype(np.uint8)
    return out, off.astype(np.uint32)


def parse(stream: np.ndarray, off: np.ndarray, N: int, K: int):
    """(positions, values) of every entry, in stream order."""
    T, W, U = shape_units(N, K)
    assert off.size == U + 1
    locs, vals = [], []
    for u in range(U):
        o = int(off[u])
        t, kc = divmod(u, W)
        h = stream[o:o + 32].view("<u4").astype(np.int64)
        n = int(h[0] >> 20)
        assert (h >> 20 == n).all()
        assert int(off[u + 1]) - o == (32 + 9 * n + 15) // 16 * 16
        v = stream[o + 32:o + 32 + 8 * n].view(np.float16).reshape(n, 4)
        k = stream[o + 32 + 8 * n:o + 32 + 9 * n].astype(np.int64)
        assert not stream[o + 32 + 9 * n:int(off[u + 1])].any()
        start = 0
        for r in range(8):
            lo, hi = int(h[r] & 1023), int((h[r] >> 10) & 1023)
            assert lo == start and hi >= lo
            for e in range(lo, hi):
                locs.append((8 * t + r) * K + 64 * kc + int(k[e]))
                vals.append(v[e])
            start = hi
        assert start == n
    return np.array(locs, dtype=np.int64), np.array(vals, dtype=np.float16).reshape(-1, 4)


def correction(stream: np.ndarray, off: np.ndarray, N: int, K: int, x: np.ndarray) -> np.ndarray:
    """corr[q][n] = sum of value_q * x[k] over the plug entries of row n (FP64)."""
    loc, v = parse(stream, off, N, K)
    corr = np.zeros((4, N))
    np.add.at(corr.T, loc // K, v.astype(np.float64) * x.astype(np.float64)[loc % K, None])
    return corr
