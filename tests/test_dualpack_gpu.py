"""``.dualpack`` streams on the GPU.

* The GPU restore of the reference-written ``dualpack_small`` stream (two
  models of unequal length, plugs, several chunks) equals the reference's
  own ``unpack_dual_models`` output bit for bit (polar_bitpack.py:194-260).
* A Linear served straight from the file layout matches the FP16 weights the
  reference installs (the restore rounded to FP16, polar_packer.py:309-310)
  times x, in float64, within 1e-3 -- on the golden stream and on a larger
  oracle-written stream with the benchmark distribution.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import formats as of
from oracle import quad as oq

pytestmark = pytest.mark.gpu
TOL = 1e-3


def test_restore_bit_exact_with_reference(cuda, dualpack_golden):
    from polar_pack_b200.dualpack import DualPackDevice, DualPackFile
    g = dualpack_golden
    pk = DualPackDevice(DualPackFile(g["stream"].tobytes()), cuda)
    w1, w2 = pk.restore()
    np.testing.assert_array_equal(w1.cpu().numpy().view(np.uint32), g["restored1"].view(np.uint32))
    np.testing.assert_array_equal(w2.cpu().numpy().view(np.uint32), g["restored2"].view(np.uint32))
    # a mid-stream range, FP16 output
    h1, h2 = pk.unpack(3000, 7001, fp16=True)
    np.testing.assert_array_equal(h1.cpu().numpy(), g["restored1"][3000:7001].astype(np.float16))


def _check_linear(pk, restored, offset, N, K, M, seed):
    lin = pk.linear(offset, N, K)
    x = np.random.default_rng(seed).normal(0, 1, size=(M, K)).astype(np.float16)
    y1, y2 = lin(torch.from_numpy(x).to(pk.device))
    for y, w in ((y1, restored[0]), (y2, restored[1])):
        W = w[offset:offset + N * K].reshape(N, K).astype(np.float16).astype(np.float64)
        ref = x.astype(np.float64) @ W.T
        assert oq.rel_err(y.cpu().numpy(), ref) <= TOL, (offset, N, K, M)


@pytest.mark.parametrize("offset,N,K,M", [(0, 40, 64, 1), (1000, 33, 128, 3), (4090, 12, 100, 2), (7, 5, 600, 4)])
def test_file_linear_golden_stream(cuda, dualpack_golden, offset, N, K, M):
    from polar_pack_b200.dualpack import DualPackDevice, DualPackFile
    g = dualpack_golden
    pk = DualPackDevice(DualPackFile(g["stream"].tobytes()), cuda)
    w = [np.pad(g["restored1"], (0, 10_000 - g["restored1"].size)), np.pad(g["restored2"], (0, 10_000 - g["restored2"].size))]
    if offset + N * K > min(g["restored1"].size, g["restored2"].size):
        pytest.skip("Linear beyond the shorter model")
    _check_linear(pk, w, offset, N, K, M, seed=offset + N)
    # the restore stays exact after the Linear cleared its plugged amplitudes
    w1, _ = pk.restore()
    np.testing.assert_array_equal(w1.cpu().numpy().view(np.uint32), g["restored1"].view(np.uint32))


def test_file_linear_benchmark_shape(cuda):
    from polar_pack_b200.dualpack import DualPackDevice, DualPackFile
    rng = np.random.default_rng(1)
    n = 2048 * 2048
    base = rng.normal(0, 0.02, n)
    w = [(base + rng.normal(0, 0.002, n)).astype(np.float16).astype(np.float32) for _ in range(2)]
    for x in w:
        idx = rng.integers(0, n, n // 1000)
        x[idx] *= 20
    buf = of.pack_dual_bytes(w[0], w[1], chunk_size=1_000_000)
    restored = of.unpack_dual_bytes(buf)
    pk = DualPackDevice(DualPackFile(buf), cuda)
    _check_linear(pk, restored, 0, 2048, 2048, 1, seed=5)
