"""Prepared tables: ``pp_quad_prepare_tables`` writes the replicated table
image, and the ``*_prepared`` entry points (bulk-copied tables) give results
bit-identical to the entry points that build the tables in the kernel."""
import ctypes

import numpy as np
import pytest
import torch

from conftest import bits
from polar_pack_b200 import _lib

pytestmark = pytest.mark.gpu


def _luts(seed, dev):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return [torch.rand(256, generator=g).half().to(dev)] + \
           [(torch.rand(256, generator=g) * 2 - 1).half().to(dev) for _ in range(6)]


def test_table_image_layout(cuda):
    luts = _luts(1, cuda)
    img = _lib.prepare_tables(luts, cuda).cpu().numpy().view(np.uint32)
    raw = [t.cpu().numpy().view(np.uint16).astype(np.uint32) for t in luts]
    words = [raw[0] | (raw[0] << 16)] + [raw[2 * t - 1] | (raw[2 * t] << 16) for t in (1, 2, 3)]
    for t in range(4):
        base = (t >> 1) * 65536 + (t & 1) * 128            # bytes: 64 KiB region, 128-byte slot
        for e in (0, 1, 77, 255):
            row = img[(base + e * 256) // 4:(base + e * 256) // 4 + 32]
            assert np.all(row == words[t][e]), (t, e)


def _gemm(fn, cuda, x, codes_v, luts_or_tables, M, N, K):
    L = _lib.load()
    outs = [torch.full((M, N), float("nan"), dtype=torch.half, device=cuda) for _ in range(4)]
    nb = ctypes.c_size_t()
    _lib.check(L.pp_quad_gemm_workspace_bytes(M, N, K, codes_v.stride(0), codes_v.stride(1), ctypes.byref(nb)))
    ws = torch.zeros(nb.value + 256, dtype=torch.uint8, device=cuda)
    tab = _lib.ptrs(luts_or_tables, 7) if fn == "pp_quad_gemm" else luts_or_tables.data_ptr()
    _lib.call(fn, x.data_ptr(), x.stride(0), x.stride(1), codes_v.data_ptr(), codes_v.stride(0),
              codes_v.stride(1), tab, _lib.floats4([0.5, 1, 2, 0.25]), _lib.ptrs(outs, 4), outs[0].stride(0),
              outs[0].stride(1), M, N, K, ws.data_ptr(), nb.value, _lib.stream_handle(cuda))
    torch.cuda.synchronize()
    return [o.cpu().numpy() for o in outs]


@pytest.mark.parametrize("layout,M,K,N", [("nk", 1, 2048, 11008), ("nk", 9, 1024, 520), ("kn", 3, 512, 2048),
                                          ("kn", 12, 300, 96), ("strided", 2, 130, 70)])
def test_prepared_equals_in_kernel_tables(cuda, layout, M, K, N):
    g = torch.Generator(device="cpu").manual_seed(M * 131 + K + N)
    luts = _luts(7, cuda)
    tables = _lib.prepare_tables(luts, cuda)
    codes = torch.randint(-2**31, 2**31 - 1, (N, K) if layout != "kn" else (K, N), generator=g,
                          dtype=torch.int32).to(cuda)
    if layout == "nk":
        cv = codes.t()
    elif layout == "kn":
        cv = codes
    else:
        cv = torch.randint(-2**31, 2**31 - 1, (K, 2 * N), generator=g, dtype=torch.int32).to(cuda)[:, ::2]
    x = torch.randn(M, K, generator=g).half().to(cuda)
    ref = _gemm("pp_quad_gemm", cuda, x, cv, luts, M, N, K)
    got = _gemm("pp_quad_gemm_prepared", cuda, x, cv, tables, M, N, K)
    for a, b in zip(ref, got):
        assert not np.isnan(b.astype(np.float32)).any()
        np.testing.assert_array_equal(bits(a), bits(b))


def test_quad_bitpacked_cache_follows_in_place_table_change(cuda):
    from polar_pack_b200.quad_kernels import pack_quad_layer, quad_bitpacked
    g = torch.Generator(device="cpu").manual_seed(5)
    ws = [(torch.randn(256, 384, generator=g) * 0.02).half().to(cuda) for _ in range(4)]
    codes, luts, scales = pack_quad_layer(*ws)
    a = torch.randn(2, 256, generator=g).half().to(cuda)
    y0 = quad_bitpacked(a, codes, luts, scales)
    luts[3].mul_(0.5)                                   # in place: version counter moves
    y1 = quad_bitpacked(a, codes, luts, scales)
    ref = quad_bitpacked(a, codes, [t.clone() for t in luts], scales)
    for k in range(4):
        assert torch.equal(y1[k], ref[k])
    assert not all(torch.equal(y0[k], y1[k]) for k in range(4))


def test_linear_prepared_equals_in_kernel_tables(cuda):
    """File-layout Linear with plugs: pp_quad_linear vs pp_quad_linear_prepared."""
    from oracle import formats as of
    from polar_pack_b200.quadpack import QuadPackDevice, QuadPackFile
    rng = np.random.default_rng(3)
    N, K = 300, 512
    base = rng.normal(0, 0.02, size=N * K)
    models = []
    for _ in range(4):
        w = base + rng.normal(0, 0.002, size=N * K)
        idx = rng.choice(w.size, size=w.size // 1000, replace=False)
        w[idx] *= 20
        models.append(w.astype(np.float16).astype(np.float32))
    pk = QuadPackDevice(QuadPackFile(of.pack_quad_bytes(models, plug_cap=0.05, threshold_windows=8, window=4096)),
                        cuda)
    lin = pk.linear(0, N, K)
    assert lin.p_hi > lin.p_lo
    for M in (1, 5):
        x = torch.randn(M, K, generator=torch.Generator().manual_seed(M)).half().to(cuda)
        res = []
        for fn, tab in (("pp_quad_linear", _lib.ptrs(pk.luts, 7)), ("pp_quad_linear_prepared", pk.tables.data_ptr())):
            outs = [torch.empty((M, N), dtype=torch.half, device=cuda) for _ in range(4)]
            nb = ctypes.c_size_t()
            _lib.check(_lib.load().pp_quad_linear_workspace_bytes(M, N, K, ctypes.byref(nb)))
            ws = torch.zeros(nb.value + 256, dtype=torch.uint8, device=cuda)
            _lib.call(fn, x.data_ptr(), x.stride(0), x.stride(1), lin.codes.data_ptr(), K, lin.plug_idx.data_ptr(),
                      lin.plug_vals.data_ptr(), lin.plug_window_base.data_ptr(), ctypes.c_uint32(0), tab,
                      _lib.floats4(pk.scales), _lib.ptrs(outs, 4), outs[0].stride(0), outs[0].stride(1), M, N, K,
                      ws.data_ptr(), nb.value, _lib.stream_handle(cuda))
            torch.cuda.synchronize()
            res.append([o.cpu().numpy() for o in outs])
        for a, b in zip(*res):
            np.testing.assert_array_equal(bits(a), bits(b))
