"""Per-model FP16 tails on the GPU: Linears that reach past ``n_min``.

The stream is the reference-written ``quadpack_small`` (four models of
unequal length: tails of 0 / 40 / 0 / 17 weights, reference
quaternion_packer.py:118-126).  A Linear whose range crosses ``n_min`` runs
its coded rows on the fused quad kernel, the row cut by ``n_min`` from the
assembled unpack + tail, and the rows past ``n_min`` on ``pp_f16_linear``
over the tails in place.  The oracle is the restore of
quaternion_packer.py:141-214 on the FP16 tables: coded positions decoded
(plug values substituted) times ``s_k``, tail positions raw FP16
(201-210); then a float64 matmul.  Models too short for a Linear get None.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import formats as of
from oracle import quad as oq

pytestmark = pytest.mark.gpu
TOL = 1e-3


def oracle_model_weights(buf, k, offset, N, K):
    """Model k's (N, K) weights at flat ``offset`` as float64, FP16-table decode."""
    hdr, codes, pidx, pval, tails = of.quad_sections(buf)
    n = hdr["n"]
    end = offset + N * K
    w = np.empty(N * K, dtype=np.float64)
    c_hi = min(end, n)
    if offset < n:
        dec = oq.decode_quad_fp16(codes[offset:c_hi], oq.quad_luts(hdr["r_max"]))[k].astype(np.float64)
        sel = (pidx >= offset) & (pidx < c_hi)
        dec[pidx[sel].astype(np.int64) - offset] = pval[sel, k].astype(np.float64)
        # one FP16 rounding of w * s_k, as the unpack of the cut row stores it
        w[:c_hi - offset] = dec * hdr["scales"][k]
    if end > n:
        lo = max(offset, n)
        w[lo - offset:] = tails[k][lo - n:end - n].astype(np.float64)
    return w.reshape(N, K)


# (offset relative to n_min, N, K): coded rows + a cut row + tail rows;
# rows exactly meeting n_min; wholly inside the tails; several batch rows; an
# offset that is not a multiple of 4 codes (the coded rows get an aligned copy)
CASES = [(-20, 7, 8, 1), (-19, 3, 12, 1), (-12, 7, 4, 2), (8, 4, 8, 1), (-4090, 129, 32, 3), (-4092, 129, 32, 3),
         (0, 5, 4, 1)]


@pytest.mark.parametrize("rel,N,K,M", CASES)
def test_tailed_linear_matches_oracle(cuda, quadpack_small_stream, rel, N, K, M):
    from polar_pack_b200.quadpack import QuadPackDevice, QuadPackFile, QuadTailedLinear
    buf = quadpack_small_stream
    pk = QuadPackDevice(QuadPackFile(buf), cuda)
    n = pk.header.n
    offset = n + rel
    lin = pk.linear(offset, N, K)
    assert isinstance(lin, QuadTailedLinear)
    x = np.random.default_rng(N * K + M).normal(0, 1, size=(M, K)).astype(np.float16)
    ys = lin(torch.from_numpy(x).to(cuda))
    torch.cuda.synchronize()
    end = offset + N * K
    for k in range(4):
        if end > pk.model_length(k):
            assert ys[k] is None, k
            continue
        w = oracle_model_weights(buf, k, offset, N, K)
        ref = x.astype(np.float64) @ w.T
        got = ys[k].cpu().numpy()
        assert oq.rel_err(got, ref) <= TOL, (k, oq.rel_err(got, ref))
    # the Linear is kept: a second request gives the same object
    assert pk.linear(offset, N, K) is lin


def test_tailed_linear_against_reference_restore(cuda, quadpack_small_stream, quadpack_golden):
    """Rows wholly inside model 1's tail against the reference's own
    ``unpack_quad`` output recorded in the fixture (raw FP16 tails)."""
    from polar_pack_b200.quadpack import QuadPackDevice, QuadPackFile
    pk = QuadPackDevice(QuadPackFile(quadpack_small_stream), cuda)
    n = pk.header.n
    lin = pk.linear(n, 5, 8)                  # model 1's 40 tail weights
    x = np.random.default_rng(3).normal(0, 1, size=(1, 8)).astype(np.float16)
    ys = lin(torch.from_numpy(x).to(cuda))
    w = quadpack_golden["tail_restored1"].reshape(5, 8).astype(np.float64)
    ref = x.astype(np.float64) @ w.T
    assert ys[0] is None and ys[2] is None and ys[3] is None
    assert oq.rel_err(ys[1].cpu().numpy(), ref) <= TOL


def test_linear_past_every_model_rejected(cuda, quadpack_small_stream):
    from polar_pack_b200.quadpack import QuadPackDevice, QuadPackFile
    pk = QuadPackDevice(QuadPackFile(quadpack_small_stream), cuda)
    with pytest.raises(ValueError):
        pk.linear(pk.header.n + 8, 5, 8)      # ends at n + 48 > n + 40
