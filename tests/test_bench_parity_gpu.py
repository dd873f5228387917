"""Oracle parity at the configurations ``bench.py`` times.

* The single-layer sweep: Linear in x out 2048x2048,
  2048x11008, 11008x2048, 2048x256 at batch 1, on one ``.quadpack`` stream
  written by the oracle writer (which reproduces the reference writer byte
  for byte) from models of the benchmark distribution, served by
  ``QuadPackDevice.linear`` + ``quad_linear`` exactly as the bench serves
  them (the fused plug-correcting GEMV).  Every output row of every model is
  compared with the oracle: FP16-table decode (quad_kernels.py:103-121) with
  the plug values substituted (quaternion_packer.py:187-193), float64
  matmul, FP32 scale, FP16 rounding.
* The batched rows of configs[3] on the two large sweep shapes at 16, 32 and
  64 rows (above 16 rows: the tcgen05 kernel with its plug correction).
* The decode-step shapes of configs[2]: qkv 2560x2048, gate_up 22016x2048
  (every row), and the lm_head 151936x2048, whose batch-1 launch runs in row
  chunks (sampled rows from every part of it).

Tolerance: max|y - y_ref| / max|y_ref| <= 1e-3 per output vector.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import formats as of
from oracle import quad as oq

pytestmark = pytest.mark.gpu
TOL = 1e-3
SWEEP = [(2048, 2048), (2048, 11008), (11008, 2048), (2048, 256)]  # (in K, out N)


def bench_models(n: int, seed: int) -> list[np.ndarray]:
    """Four correlated models: base N(0,0.02) + delta N(0,0.002), 0.1% x20, FP16."""
    rng = np.random.default_rng(seed)
    base = rng.normal(0, 0.02, n).astype(np.float32)
    out = []
    for _ in range(4):
        w = base + rng.normal(0, 0.002, n).astype(np.float32)
        idx = rng.integers(0, n, n // 1000)
        w[idx] *= 20
        out.append(w.astype(np.float16).astype(np.float32))
    return out


@pytest.fixture(scope="module")
def sweep(cuda):
    from polar_pack_b200.quadpack import QuadPackDevice, QuadPackFile
    n = sum(K * N for K, N in SWEEP)
    buf = of.pack_quad_bytes(bench_models(n, 0), plug_cap=0.05, threshold_windows=8, window=1_000_000)
    hdr, codes, pidx, pval, _ = of.quad_sections(buf)
    pk = QuadPackDevice(QuadPackFile(buf), cuda)
    offs, o = [], 0
    for K, N in SWEEP:
        offs.append(o)
        o += K * N
    return dict(buf=buf, hdr=hdr, codes=codes, pidx=pidx, pval=pval, pk=pk, offs=offs)


def oracle_rows(sw, offset, N, K):
    """(4, N, K) FP16 weights of the Linear: decode with plugs substituted."""
    c = sw["codes"][offset:offset + N * K].reshape(N, K)
    w = oq.decode_quad_fp16(c, oq.quad_luts(sw["hdr"]["r_max"]))
    sel = (sw["pidx"] >= offset) & (sw["pidx"] < offset + N * K)
    loc = sw["pidx"][sel].astype(np.int64) - offset
    for k in range(4):
        w[k].reshape(-1)[loc] = sw["pval"][sel, k]
    return w


def check(y, x, w, scales, what):
    """y: (4, M, N) GPU result; w: (4, N, K) FP16 weights."""
    ref = oq.quad_gemm(x, None, None, scales, decoded=[wk.T for wk in w])
    for k in range(4):
        err = oq.rel_err(np.asarray(y[k], np.float32), ref[k])
        assert err <= TOL, (what, k, err)


@pytest.mark.parametrize("j", range(len(SWEEP)))
def test_sweep_batch1_every_row(cuda, sweep, j):
    from polar_pack_b200.quadpack import quad_linear
    K, N = SWEEP[j]
    lin = sweep["pk"].linear(sweep["offs"][j], N, K)
    assert lin.unit_plugs is not None          # the bench's fused path
    x = np.random.default_rng(j).normal(0, 1, size=(1, K)).astype(np.float16)
    y = quad_linear(torch.from_numpy(x).to(cuda), lin)
    got = torch.stack(y).cpu().numpy()
    check(got, x, oracle_rows(sweep, sweep["offs"][j], N, K), sweep["hdr"]["scales"], SWEEP[j])


@pytest.mark.parametrize("M", [16, 32, 64])
@pytest.mark.parametrize("j", [1, 2])
def test_sweep_batched_rows(cuda, sweep, j, M):
    from polar_pack_b200.quadpack import quad_linear
    K, N = SWEEP[j]
    lin = sweep["pk"].linear(sweep["offs"][j], N, K)
    x = np.random.default_rng(100 * j + M).normal(0, 1, size=(M, K)).astype(np.float16)
    y = quad_linear(torch.from_numpy(x).to(cuda), lin)
    got = torch.stack(y).cpu().numpy()
    check(got, x, oracle_rows(sweep, sweep["offs"][j], N, K), sweep["hdr"]["scales"], (SWEEP[j], M))


class DevLinear:
    """A file-layout Linear of random codes with 5% plugs, built on the GPU
    (large shapes), prepared as ``QuadPackDevice.linear`` prepares one."""

    BASE = 0x7FFFF000  # stream offset: positions cross 2^31 inside the Linear

    def __init__(self, dev, N, K, seed):
        from polar_pack_b200 import _lib
        from polar_pack_b200.quadpack import prepare_unit_plugs
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        self.N, self.K, self.dev = N, K, dev
        self.scales = [0.5, 1.0, 2.0, 0.25]
        self.codes = torch.randint(-2**31, 2**31 - 1, (N, K), generator=g, device=dev, dtype=torch.int32)
        self.raw = self.codes.clone()             # before plug preparation zeroes norm bytes
        n = N * K
        self.loc = torch.unique(torch.randint(0, n, (n // 20,), generator=g, device=dev))
        self.pidx = ((self.loc + self.BASE) & 0xFFFFFFFF).to(torch.int64).to(torch.int32)
        self.pval = torch.randn(self.loc.numel(), 4, generator=g, device=dev).half()
        self.wb = torch.empty(N * (-(-K // 64)) + 1, dtype=torch.int32, device=dev)
        bad = torch.zeros(1, dtype=torch.int32, device=dev)
        _lib.call("pp_quad_prepare_plugs", self.codes.data_ptr(), K, self.pidx.data_ptr(), 0, self.loc.numel(),
                  ctypes.c_uint32(self.BASE), N, K, self.wb.data_ptr(), bad.data_ptr(), _lib.stream_handle(dev))
        assert int(bad.item()) == 0
        self.up, self.uo = prepare_unit_plugs(self.pidx, self.pval, self.wb, self.BASE, N, K, dev)
        self.luts_h = oq.quad_luts(1.5)
        self._luts = [torch.from_numpy(t).to(dev) for t in self.luts_h]
        self.tables = _lib.prepare_tables(self._luts, dev)
        self.loc_h = self.loc.cpu().numpy()
        self.pval_h = self.pval.cpu().numpy()

    def run(self, x):
        from polar_pack_b200 import _lib
        from polar_pack_b200.quadpack import quad_linear_workspace_bytes
        M = x.shape[0]
        out = torch.empty((4, M, self.N), dtype=torch.float16, device=self.dev)
        outs = [out[k] for k in range(4)]
        nb = quad_linear_workspace_bytes(M, self.N, self.K)
        ws = torch.zeros(max(nb, 256), dtype=torch.uint8, device=self.dev)
        _lib.call("pp_quad_linear_fused", x.data_ptr(), x.stride(0), x.stride(1), self.codes.data_ptr(), self.K,
                  self.pidx.data_ptr(), self.pval.data_ptr(), self.wb.data_ptr(), ctypes.c_uint32(self.BASE),
                  self.up.data_ptr(), self.uo.data_ptr(), self.tables.data_ptr(), _lib.floats4(self.scales),
                  _lib.ptrs(outs, 4), outs[0].stride(0), outs[0].stride(1), M, self.N, self.K, ws.data_ptr(),
                  ws.numel(), _lib.stream_handle(self.dev))
        torch.cuda.synchronize(self.dev)
        return out.cpu().numpy()

    def oracle_rows(self, rows):
        """(4, len(rows), K) FP16 weights of the given rows, plugs substituted."""
        rows = np.asarray(rows, dtype=np.int64)
        c = self.raw[torch.from_numpy(rows).to(self.dev)].cpu().numpy().view(np.uint32)
        w = oq.decode_quad_fp16(c, self.luts_h)
        K = self.K
        for i, r in enumerate(rows):
            lo, hi = np.searchsorted(self.loc_h, [r * K, (r + 1) * K])
            cols = self.loc_h[lo:hi] - r * K
            for k in range(4):
                w[k][i, cols] = self.pval_h[lo:hi, k]
        return w


@pytest.mark.parametrize("N,K", [(2560, 2048), (22016, 2048)])
def test_decode_step_shapes_every_row(cuda, N, K):
    lin = DevLinear(cuda, N, K, seed=N)
    x = np.random.default_rng(N).normal(0, 1, size=(1, K)).astype(np.float16)
    got = lin.run(torch.from_numpy(x).to(cuda))
    w = lin.oracle_rows(np.arange(N))
    check(got, x, w, lin.scales, (N, K))


def test_lm_head_row_chunks(cuda):
    """151936 x 2048 at batch 1: more units than one launch's offset tables
    hold, so the fused entry launches row chunks.  4096 rows are checked:
    the first and last rows, and rows spread over the whole Linear."""
    N, K = 151936, 2048
    lin = DevLinear(cuda, N, K, seed=5)
    x = np.random.default_rng(5).normal(0, 1, size=(1, K)).astype(np.float16)
    got = lin.run(torch.from_numpy(x).to(cuda))
    rng = np.random.default_rng(6)
    rows = np.unique(np.concatenate([np.arange(64), np.arange(N - 64, N), rng.choice(N, 3968, replace=False)]))
    w = lin.oracle_rows(rows)
    check(got[:, :, rows], x, w, lin.scales, "lm_head")
    del lin
    torch.cuda.empty_cache()
