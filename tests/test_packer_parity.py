"""The product's ``.quadpack`` packer (``pack_quad_device``) against the oracle
writer, which reproduces the reference's ``pack_quad`` byte for byte
(quaternion_packer.py:52-138; test_oracle_golden.py).

The two run the same passes: float64 RMS, ``r_max * 1.001``, the
``(1 - plug_cap)`` percentile of the decode error over seeded windows, then
codes and plug entries.  The packer computes its float32 transcendentals with
torch instead of numpy, so a code whose value sits on a rounding boundary can
differ by one quantisation step in one of its four fields.  The contract
checked here: identical header (n, scales, r_max, plug count, tails),
identical plug table (positions and FP16 values), identical tails, and codes
identical except for at most 1e-4 of them, each of which differs by exactly
one step in exactly one byte.  On the GPU the float64 RMS sums reduce in
another order, which the looser GPU contract of ``compare`` allows for.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import formats as of


def models(n, seed, extra=(0, 0, 0, 0)):
    rng = np.random.default_rng(seed)
    base = rng.normal(0, 0.02, n + max(extra)).astype(np.float32)
    out = []
    for k in range(4):
        w = base + rng.normal(0, 0.002, base.size).astype(np.float32)
        idx = rng.integers(0, w.size, w.size // 1000)
        w[idx] *= 20
        out.append(w[: n + extra[k]].astype(np.float16))
    return out


def compare(ref: bytes, got: bytes, strict: bool = True):
    """``strict``: the CPU contract above.  Otherwise (GPU): the float64 RMS
    sums reduce in another order, so scales and r_max may differ in their last
    bits and the plug threshold with them; then the header agrees to 1e-12,
    the plug sets agree up to 1e-3 of their entries (values identical where
    positions agree), and the codes as on the CPU."""
    hr, cr, pir, pvr, tr = of.quad_sections(ref)
    hg, cg, pig, pvg, tg = of.quad_sections(got)
    for key in ("n", "tails", "mu", "bits"):
        assert hr[key] == hg[key], key
    if strict:
        assert len(ref) == len(got) and hr["plug_n"] == hg["plug_n"]
        assert hr["scales"] == hg["scales"] and hr["r_max"] == hg["r_max"]
        np.testing.assert_array_equal(pir, pig)
        np.testing.assert_array_equal(pvr.view(np.uint16), pvg.view(np.uint16))
    else:
        np.testing.assert_allclose(hg["scales"], hr["scales"], rtol=1e-12)
        np.testing.assert_allclose(hg["r_max"], hr["r_max"], rtol=1e-6)
        common, ir, ig = np.intersect1d(pir, pig, return_indices=True)
        assert max(pir.size, pig.size) - common.size <= max(1, pir.size // 1000)
        # the values are FP16 of w / s_k: equal unless s_k moved them across a rounding boundary
        assert np.mean(pvr[ir].view(np.uint16) == pvg[ig].view(np.uint16)) >= 0.999
    for a, b in zip(tr, tg):
        np.testing.assert_array_equal(a.view(np.uint16), b.view(np.uint16))
    d = np.nonzero(cr != cg)[0]
    assert d.size <= max(1, cr.size // 10_000), d.size
    for sh in (24, 16, 8, 0):
        diff = ((cr[d] >> sh) & 255).astype(np.int64) - ((cg[d] >> sh) & 255).astype(np.int64)
        assert np.all(np.abs(diff) <= 1)
    fields = sum(((cr[d] >> sh) & 255) != ((cg[d] >> sh) & 255) for sh in (24, 16, 8, 0))
    assert np.all(fields == 1)


def pack_both(ms, device):
    from polar_pack_b200.quadpack import pack_quad_device, to_bytes
    ref = of.pack_quad_bytes([m.astype(np.float32) for m in ms], plug_cap=0.05, threshold_windows=4,
                             window=1_000_000)
    p = pack_quad_device([torch.from_numpy(m).to(device) for m in ms], plug_cap=0.05, seed=42, windows=4,
                         window=1_000_000, chunk=1 << 20)
    return ref, to_bytes(p)


def test_device_packer_matches_oracle_writer_cpu():
    ref, got = pack_both(models(3_000_000, 0, (0, 40, 0, 17)), "cpu")
    compare(ref, got)


@pytest.mark.gpu
def test_device_packer_matches_oracle_writer_gpu(cuda):
    ref, got = pack_both(models(3_000_000, 1, (0, 0, 33, 0)), cuda)
    compare(ref, got, strict=False)
