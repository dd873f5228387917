"""Grouped launches (``pp_quad_linear_group``): several independent packed
Linears in one kernel launch, each on its share of the SMs.

* The sweep's four Linears (the benchmark's step) run as ONE launch, and each
  member's outputs match the oracle (FP16-table decode with plugs
  substituted, float64 matmul) within 1e-3; repeated launches are
  bit-identical (fixed split-K order per member).
* A group that cannot run as one launch (batch 2) runs its members one
  after another, bit-identical to separate calls.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import formats as of
from oracle import quad as oq

pytestmark = pytest.mark.gpu
TOL = 1e-3
SHAPES = [(2048, 2048), (2048, 11008), (11008, 2048), (2048, 256)]  # (K in, N out)


@pytest.fixture(scope="module")
def stream(cuda):
    from polar_pack_b200.quadpack import QuadPackDevice, QuadPackFile
    n = sum(K * N for K, N in SHAPES)
    rng = np.random.default_rng(4)
    base = rng.normal(0, 0.02, n).astype(np.float32)
    models = []
    for _ in range(4):
        w = base + rng.normal(0, 0.002, n).astype(np.float32)
        idx = rng.integers(0, n, n // 1000)
        w[idx] *= 20
        models.append(w.astype(np.float16).astype(np.float32))
    buf = of.pack_quad_bytes(models, plug_cap=0.05, threshold_windows=4, window=1_000_000)
    pk = QuadPackDevice(QuadPackFile(buf), cuda)
    layers, off = [], 0
    for K, N in SHAPES:
        layers.append(pk.linear(off, N, K))
        off += K * N
    return buf, pk, layers


def oracle_out(buf, layer, x):
    hdr, codes, pidx, pval, _ = of.quad_sections(buf)
    off, N, K = layer.offset, layer.N, layer.K
    w = oq.decode_quad_fp16(codes[off:off + N * K].reshape(N, K), oq.quad_luts(hdr["r_max"]))
    sel = (pidx >= off) & (pidx < off + N * K)
    for k in range(4):
        w[k].reshape(-1)[pidx[sel].astype(np.int64) - off] = pval[sel, k]
    return oq.quad_gemm(x, None, None, hdr["scales"], decoded=[wk.T for wk in w])


def test_sweep_as_one_launch_matches_oracle(cuda, stream):
    from polar_pack_b200.quadpack import QuadLinearGroup
    buf, pk, layers = stream
    g = torch.Generator(device=cuda).manual_seed(1)
    xs = [torch.randn(1, K, generator=g, device=cuda).half() for K, _ in SHAPES]
    outs = [[torch.full((1, N), float("nan"), dtype=torch.half, device=cuda) for _ in range(4)] for _, N in SHAPES]
    grp = QuadLinearGroup(layers, xs, outs)
    assert grp.single_launch
    grp()
    torch.cuda.synchronize()
    first = [[o.clone() for o in os_] for os_ in outs]
    for j, l in enumerate(layers):
        ref = oracle_out(buf, l, xs[j].cpu().numpy())
        for k in range(4):
            got = outs[j][k].cpu().numpy()
            assert not np.isnan(got.astype(np.float32)).any()
            assert oq.rel_err(got, ref[k]) <= TOL, (SHAPES[j], k)
    for _ in range(2):  # deterministic
        grp()
        torch.cuda.synchronize()
        for j in range(len(layers)):
            for k in range(4):
                assert torch.equal(outs[j][k].view(torch.int16), first[j][k].view(torch.int16))


def test_group_members_one_after_another(cuda, stream):
    """Two batch rows: no one-launch path; each member equals its own call."""
    from polar_pack_b200.quadpack import QuadLinearGroup, quad_linear
    _, _, layers = stream
    g = torch.Generator(device=cuda).manual_seed(2)
    xs = [torch.randn(2, K, generator=g, device=cuda).half() for K, _ in SHAPES]
    outs = [[torch.empty((2, N), dtype=torch.half, device=cuda) for _ in range(4)] for _, N in SHAPES]
    grp = QuadLinearGroup(layers, xs, outs)
    assert not grp.single_launch
    grp()
    for j, l in enumerate(layers):
        ref = quad_linear(xs[j], l)
        for k in range(4):
            assert torch.equal(outs[j][k].view(torch.int16), ref[k].view(torch.int16))


def test_per_model_rows_with_interleaved_copy(cuda, stream):
    """Per-model activation rows (model k multiplies row k, as in a 4-model
    decode step) against the oracle; with the interleaved copy x_il the plug
    correction reads its activations differently but sums the same terms in
    the same order: bit-identical."""
    from polar_pack_b200.quadpack import QuadLinearGroup
    buf, pk, layers = stream
    g = torch.Generator(device=cuda).manual_seed(3)
    xs = [torch.randn(4, K, generator=g, device=cuda).half() for K, _ in SHAPES]
    ils = [x.t().contiguous().view(-1) for x in xs]
    res = []
    for x_ils in (None, ils):
        outs = [[torch.full((1, N), float("nan"), dtype=torch.half, device=cuda) for _ in range(4)]
                for _, N in SHAPES]
        grp = QuadLinearGroup(layers, xs, outs, per_model_x=True, x_ils=x_ils)
        assert grp.single_launch
        grp()
        torch.cuda.synchronize()
        res.append(outs)
    for j, l in enumerate(layers):
        for k in range(4):
            ref = oracle_out(buf, l, xs[j][k:k + 1].cpu().numpy())
            got = res[0][j][k].cpu().numpy()
            assert oq.rel_err(got, ref[k]) <= TOL, (SHAPES[j], k)
            assert torch.equal(res[1][j][k].view(torch.int16), res[0][j][k].view(torch.int16)), (SHAPES[j], k)
