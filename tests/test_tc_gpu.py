"""Batched quad GEMM on the tcgen05 tensor cores (file layout, > 16 batch
rows, prepared tables, N >= 4096 or K >= 4096): outputs against the numpy
oracle (float64 matmul of the oracle's bit-exact FP16 decode), determinism,
the split-K partition, ragged tiles and batch rows beyond one 128-row
launch."""
import ctypes

import numpy as np
import pytest
import torch

from conftest import bits
from oracle import quad as oq
from polar_pack_b200 import _lib

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _case(K, N, seed, cuda):
    g = torch.Generator(device="cpu").manual_seed(seed)
    base = torch.randn(K, N, generator=g) * 0.02
    from polar_pack_b200.quad_kernels import pack_quad_layer
    ws = [(base + torch.randn(K, N, generator=g) * 0.002).half().to(cuda) for _ in range(4)]
    codes, luts, scales = pack_quad_layer(*ws)          # codes (K, N)
    codes_nk = codes.t().contiguous()                    # file layout [N][K]
    return codes_nk, luts, scales, g


def _run_prepared(cuda, x, codes_nk, luts, scales):
    M, K = x.shape
    N = codes_nk.shape[0]
    cv = codes_nk.t()                                    # (K, N) view, K contiguous
    outs = [torch.full((M, N), float("nan"), dtype=torch.half, device=cuda) for _ in range(4)]
    nb = ctypes.c_size_t()
    L = _lib.load()
    _lib.check(L.pp_quad_gemm_workspace_bytes(M, N, K, cv.stride(0), cv.stride(1), ctypes.byref(nb)))
    ws = torch.zeros(nb.value + 256, dtype=torch.uint8, device=cuda)
    tables = _lib.prepare_tables(luts, cuda)
    _lib.call("pp_quad_gemm_prepared", x.data_ptr(), x.stride(0), x.stride(1), cv.data_ptr(), cv.stride(0),
              cv.stride(1), tables.data_ptr(), _lib.floats4(scales), _lib.ptrs(outs, 4), outs[0].stride(0),
              outs[0].stride(1), M, N, K, ws.data_ptr(), nb.value, _lib.stream_handle(cuda))
    torch.cuda.synchronize()
    return [o.cpu().numpy() for o in outs]


# shapes the tensor-core path takes (N >= 4096 or K >= 4096): ragged last
# tile (N % 128), more than 128 batch rows (two launches), split-K
@pytest.mark.parametrize("M,K,N", [(17, 4096, 128), (32, 4096, 384), (64, 4096, 520), (40, 1024, 4224),
                                   (128, 4096, 256), (130, 4096, 136)])
def test_tc_matches_oracle(cuda, M, K, N):
    codes_nk, luts, scales, g = _case(K, N, M * 7 + K + N, cuda)
    x = torch.randn(M, K, generator=g).half()
    got = _run_prepared(cuda, x.to(cuda), codes_nk, luts, scales)
    ref = oq.quad_gemm(x.numpy(), codes_nk.t().cpu().numpy(), [t.cpu().numpy() for t in luts], scales)
    for k in range(4):
        assert not np.isnan(got[k].astype(np.float32)).any(), k
        assert oq.rel_err(got[k], ref[k]) <= TOL, (k, oq.rel_err(got[k], ref[k]))


def test_tc_deterministic_and_split_k(cuda):
    # 4096 in x 2048 out at 64 rows: 16 tiles, split-K across CTAs
    codes_nk, luts, scales, g = _case(4096, 2048, 3, cuda)
    x = torch.randn(64, 4096, generator=g).half().to(cuda)
    a = _run_prepared(cuda, x, codes_nk, luts, scales)
    b = _run_prepared(cuda, x, codes_nk, luts, scales)
    for k in range(4):
        np.testing.assert_array_equal(bits(a[k]), bits(b[k]))
    ref = oq.quad_gemm(x.cpu().numpy(), codes_nk.t().cpu().numpy(), [t.cpu().numpy() for t in luts], scales)
    for k in range(4):
        assert oq.rel_err(a[k], ref[k]) <= TOL
