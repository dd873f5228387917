"""GPU parity of the plug correction fused into the quad GEMV.

The device builder of the unit-major plug stream must equal the numpy
writer byte for byte; ``pp_quad_linear_fused`` at batch 1 must match the
oracle (FP16 decode with the plug values substituted) within the output
tolerance, including units too large for their shared-memory plug slot,
rows without plugs and ragged shapes; and larger batches or partitions too
long for the warps' offset tables must take the separate correction kernel.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import unit_plugs_ref as upr
from oracle import quad as oq

pytestmark = pytest.mark.gpu
TOL = 1e-3
BASE = 0xFFFF0000  # stream offset of the Linear: positions wrap past 2^32


class Linear:
    """One synthetic file-layout Linear with its plug table on the GPU."""

    def __init__(self, dev, N, K, density, cluster, seed):
        from polar_pack_b200 import _lib
        from polar_pack_b200.quadpack import prepare_unit_plugs
        rng = np.random.default_rng(seed)
        self.N, self.K, self.dev = N, K, dev
        self.codes_h = rng.integers(0, 2**32, size=(N, K), dtype=np.uint64).astype(np.uint32)
        self.loc, self.vals = upr.random_plugs(rng, N, K, density, cluster)
        self.luts_h = oq.quad_luts(1.5)
        self.scales = [0.5, 1.0, 2.0, 0.25]
        self.codes = torch.from_numpy(self.codes_h.view(np.int32)).to(dev)
        pos = ((self.loc + BASE) & 0xFFFFFFFF).astype(np.uint32)
        self.pidx = torch.from_numpy(pos.view(np.int32)).to(dev)
        self.pval = torch.from_numpy(self.vals).to(dev)
        W = -(-K // 64)
        self.wb = torch.empty(N * W + 1, dtype=torch.int32, device=dev)
        bad = torch.zeros(1, dtype=torch.int32, device=dev)
        P = self.loc.size
        _lib.call("pp_quad_prepare_plugs", self.codes.data_ptr(), K, self.pidx.data_ptr(), 0, P,
                  ctypes.c_uint32(BASE), N, K, self.wb.data_ptr(), bad.data_ptr(), _lib.stream_handle(dev))
        assert int(bad.item()) == 0
        self.up, self.uo = prepare_unit_plugs(self.pidx, self.pval, self.wb, BASE, N, K, dev)
        luts = [torch.from_numpy(t).to(dev) for t in self.luts_h]
        self._luts = luts
        self.tables = _lib.prepare_tables(luts, dev)

    def oracle_weights(self):
        w = oq.decode_quad_fp16(self.codes_h, self.luts_h)
        for k in range(4):
            flat = w[k].reshape(-1)
            flat[self.loc] = self.vals[:, k]
        return w

    def run(self, x, entry="pp_quad_linear_fused", wb=None):
        from polar_pack_b200 import _lib
        from polar_pack_b200.quadpack import quad_linear_workspace_bytes
        M = x.shape[0]
        out = torch.empty((4, M, self.N), dtype=torch.float16, device=self.dev)
        outs = [out[k] for k in range(4)]
        nb = quad_linear_workspace_bytes(M, self.N, self.K)
        ws = torch.zeros(max(nb, 256), dtype=torch.uint8, device=self.dev)
        wbp = (wb if wb is not None else self.wb).data_ptr()
        head = (x.data_ptr(), x.stride(0), x.stride(1), self.codes.data_ptr(), self.K, self.pidx.data_ptr(),
                self.pval.data_ptr(), wbp, ctypes.c_uint32(BASE))
        if entry == "pp_quad_linear_fused":  # a Linear without plugs passes no unit plugs
            has = self.pval.numel() > 0
            head = head + ((self.up.data_ptr(), self.uo.data_ptr()) if has else (None, None))
        _lib.call(entry, *head, self.tables.data_ptr(), _lib.floats4(self.scales), _lib.ptrs(outs, 4),
                  outs[0].stride(0), outs[0].stride(1), M, self.N, self.K, ws.data_ptr(), ws.numel(),
                  _lib.stream_handle(self.dev))
        torch.cuda.synchronize(self.dev)
        return out.cpu().numpy()


CASES = [  # (N, K, density, cluster)
    (8, 64, 0.05, False),
    (13, 100, 0.05, False),
    (256, 2048, 0.05, True),
    (2048, 256, 0.05, True),
    (1000, 1028, 0.02, True),
    (64, 4096, 0.10, False),
    (24, 192, 0.0, False),
]


@pytest.mark.parametrize("N,K,density,cluster", CASES)
def test_unit_stream_matches_numpy(cuda, N, K, density, cluster):
    lin = Linear(cuda, N, K, density, cluster, seed=N + 3 * K)
    stream, off = upr.build(lin.loc, lin.vals, N, K)
    uo = lin.uo.cpu().numpy().view(np.uint32)
    assert np.array_equal(uo, off)
    got = lin.up.cpu().numpy()[: int(off[-1])]
    assert np.array_equal(got, stream)


def check_against_oracle(lin, y, x):
    w = lin.oracle_weights()
    ref = oq.quad_gemm(x, None, None, lin.scales, decoded=[wk.T for wk in w])
    for k in range(4):
        err = oq.rel_err(y[k], ref[k])
        assert err <= TOL, (lin.N, lin.K, x.shape[0], k, err)


@pytest.mark.parametrize("N,K,density,cluster", CASES)
def test_fused_batch1_matches_oracle(cuda, N, K, density, cluster):
    lin = Linear(cuda, N, K, density, cluster, seed=11 * N + K)
    x = np.random.default_rng(5).normal(0, 1, size=(1, K)).astype(np.float16)
    y = lin.run(torch.from_numpy(x).to(cuda))
    check_against_oracle(lin, y, x)


@pytest.mark.parametrize("N,K,density,cluster", CASES[2:6])
def test_fused_path_taken_at_batch1(cuda, N, K, density, cluster):
    """With a zeroed window index the separate correction kernel would add
    nothing; a correct batch-1 result shows that the fused path ran."""
    lin = Linear(cuda, N, K, density, cluster, seed=N + K)
    x = np.random.default_rng(6).normal(0, 1, size=(1, K)).astype(np.float16)
    y = lin.run(torch.from_numpy(x).to(cuda), wb=torch.zeros_like(lin.wb))
    check_against_oracle(lin, y, x)


def test_fused_deterministic(cuda):
    lin = Linear(cuda, 2048, 2048, 0.05, True, seed=1)
    xd = torch.from_numpy(np.random.default_rng(2).normal(0, 1, size=(1, 2048)).astype(np.float16)).to(cuda)
    a = lin.run(xd)
    for _ in range(3):
        assert np.array_equal(lin.run(xd).view(np.uint16), a.view(np.uint16))


@pytest.mark.parametrize("M", [2, 5, 16, 40])
def test_fused_entry_larger_batch(cuda, M):
    """Batches above one row take the separate correction kernel."""
    lin = Linear(cuda, 200, 1024, 0.05, True, seed=M)
    x = np.random.default_rng(M).normal(0, 1, size=(M, 1024)).astype(np.float16)
    y = lin.run(torch.from_numpy(x).to(cuda))
    check_against_oracle(lin, y, x)


def test_fused_close_to_unfused(cuda):
    lin = Linear(cuda, 1024, 4096, 0.05, False, seed=3)
    xd = torch.from_numpy(np.random.default_rng(4).normal(0, 1, size=(1, 4096)).astype(np.float16)).to(cuda)
    a = lin.run(xd).astype(np.float32)
    b = lin.run(xd, entry="pp_quad_linear_prepared").astype(np.float32)
    for k in range(4):
        assert oq.rel_err(a[k], b[k]) <= TOL


def test_long_partition_runs_in_row_chunks(cuda):
    """8192 x 16384 gives each warp about 110 units, more than its offset
    table holds: the fused entry then launches row chunks that fit.  With a
    zeroed window index the separate correction kernel would add nothing, so
    agreement with the unfused path shows that the chunks ran fused."""
    from polar_pack_b200 import _lib
    from polar_pack_b200.quadpack import prepare_unit_plugs

    class Big(Linear):
        def __init__(self, dev, N, K):
            g = torch.Generator(device=dev)
            g.manual_seed(0)
            self.N, self.K, self.dev = N, K, dev
            self.scales = [0.5, 1.0, 2.0, 0.25]
            self.codes = torch.randint(-2**31, 2**31 - 1, (N, K), generator=g, device=dev, dtype=torch.int32)
            n = N * K
            loc = torch.unique(torch.randint(0, n, (n // 100,), generator=g, device=dev))
            self.pidx = ((loc + BASE) & 0xFFFFFFFF).to(torch.int64).to(torch.int32)
            self.pval = torch.randn(loc.numel(), 4, generator=g, device=dev).half()
            self.wb = torch.empty(N * (-(-K // 64)) + 1, dtype=torch.int32, device=dev)
            _lib.call("pp_quad_prepare_plugs", self.codes.data_ptr(), K, self.pidx.data_ptr(), 0, loc.numel(),
                      ctypes.c_uint32(BASE), N, K, self.wb.data_ptr(), None, _lib.stream_handle(dev))
            self.up, self.uo = prepare_unit_plugs(self.pidx, self.pval, self.wb, BASE, N, K, dev)
            self._luts = [torch.from_numpy(t).to(dev) for t in oq.quad_luts(1.5)]
            self.tables = _lib.prepare_tables(self._luts, dev)

    lin = Big(cuda, 8192, 16384)
    xd = torch.randn(1, 16384, device=cuda).half()
    a = lin.run(xd, wb=torch.zeros_like(lin.wb)).astype(np.float32)
    b = lin.run(xd, entry="pp_quad_linear_prepared").astype(np.float32)
    for k in range(4):
        assert oq.rel_err(a[k], b[k]) <= TOL, k
    del lin
    torch.cuda.empty_cache()


@pytest.mark.parametrize("M", [3, 17, 33, 64, 130])
def test_batched_plugs_tensor_core_path(cuda, M):
    """N >= 4096 above 16 rows takes the tcgen05 kernel.  A launch of more
    than 32 rows substitutes the plug values into its decoded tiles; up to
    32 rows a separate kernel computes the correction for all of the
    launch's rows over the transposed activations.  130 rows are launches of
    128 (substituted) and 2 (corrected)."""
    lin = Linear(cuda, 4096, 320, 0.05, True, seed=100 + M)
    x = np.random.default_rng(M).normal(0, 1, size=(M, 320)).astype(np.float16)
    y = lin.run(torch.from_numpy(x).to(cuda))
    check_against_oracle(lin, y, x)
