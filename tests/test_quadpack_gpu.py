"""GPU parity of the file-layout path: ``.quadpack`` streams, plug merge, fused Linear.

Streams are written by the oracle's ``.quadpack`` writer, which reproduces
the reference writer byte for byte (test_oracle_golden.py).  The oracle
decodes each Linear with the FP16 tables rebuilt from the header and
substitutes plug values before the dot product.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bits
from oracle import formats as of
from oracle import quad as oq

pytestmark = pytest.mark.gpu
TOL = 1e-3

# (out, in) Linears in stream order; K % 4 == 0 for the file layout
LAYERS = [(64, 128), (40, 64), (96, 256), (8, 1024), (200, 68), (33, 132)]


@pytest.fixture(scope="module")
def stream():
    rng = np.random.default_rng(123)
    n = sum(o * i for o, i in LAYERS)
    base = rng.normal(0, 0.02, size=n + 50)
    models = []
    for k, extra in enumerate([0, 50, 0, 9]):
        w = base[: n + extra] + rng.normal(0, 0.002, size=n + extra)
        idx = rng.choice(w.size, size=w.size // 1000, replace=False)
        w[idx] *= 20
        models.append(w.astype(np.float16).astype(np.float32))
    return of.pack_quad_bytes(models, plug_cap=0.05, threshold_windows=8, window=4096)


def oracle_linear_weights(buf, offset, N, K):
    """(4 x FP16 (N, K)) decode with plugs substituted, normalised weights."""
    hdr, codes, pidx, pval, _ = of.quad_sections(buf)
    luts = oq.quad_luts(hdr["r_max"])
    c = codes[offset:offset + N * K].reshape(N, K)
    w = oq.decode_quad_fp16(c, luts)
    sel = (pidx >= offset) & (pidx < offset + N * K)
    loc = pidx[sel].astype(np.int64) - offset
    for k in range(4):
        flat = w[k].reshape(-1)
        flat[loc] = pval[sel, k]
    return w, hdr["scales"]


def test_fused_linear_matches_oracle(cuda, stream):
    from polar_pack_b200.quadpack import QuadPackDevice, QuadPackFile
    pk = QuadPackDevice(QuadPackFile(stream), cuda)
    rng = np.random.default_rng(9)
    off = 0
    n_plugged = 0
    for (N, K) in LAYERS:
        layer = pk.linear(off, N, K)
        n_plugged += layer.p_hi - layer.p_lo
        w, scales = oracle_linear_weights(stream, off, N, K)
        for M in (1, 3, 8, 12):
            x = rng.normal(0, 1, size=(M, K)).astype(np.float16)
            ys = layer(torch.from_numpy(x).to(cuda))
            ref = oq.quad_gemm(x, None, None, scales, decoded=[wk.T for wk in w])
            for k in range(4):
                assert oq.rel_err(ys[k].cpu().numpy(), ref[k]) <= TOL, (N, K, M, k)
        off += N * K
    pk.check_plug_index()
    assert n_plugged > 0


def test_gpu_unpack_bit_exact(cuda, stream):
    from polar_pack_b200.quadpack import QuadPackDevice, QuadPackFile
    pk = QuadPackDevice(QuadPackFile(stream), cuda)
    hdr, codes, pidx, pval, _ = of.quad_sections(stream)
    luts = oq.quad_luts(hdr["r_max"])
    ref = oq.decode_quad_fp16(codes, luts)
    for k in range(4):
        ref[k] = ref[k].copy()
        ref[k][pidx.astype(np.int64)] = pval[:, k]
    got = pk.unpack(scaled=False)
    for k in range(4):
        np.testing.assert_array_equal(bits(got[k].cpu().numpy()), bits(ref[k]))
    # scaled restore vs the reference float64 unpack: quantisation-level agreement
    rest = of.unpack_quad_bytes(stream)
    got = pk.unpack(scaled=True)
    for k in range(4):
        y = got[k].cpu().numpy().astype(np.float64)
        r = rest[k][: hdr["n"]].astype(np.float64)
        cos = float(y @ r / np.sqrt((y @ y) * (r @ r)))
        assert cos > 0.9999
    # a sub-range starting mid-stream uses the plug entries of that range only
    lo, hi = 1000, 5000
    part = pk.unpack(lo, hi, scaled=False)
    for k in range(4):
        np.testing.assert_array_equal(bits(part[k].cpu().numpy()), bits(ref[k][lo:hi]))

