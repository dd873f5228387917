"""GPU parity of the quad kernel (drop-in ``quad_bitpacked`` / ``quad_decode``).

Bar: decoded FP16 weights bit-exact with the oracle's FP16 chain given the
same tables; outputs within ``max|y - y_ref| / max|y_ref| <= 1e-3`` per output
vector (FP32 accumulation order differs from the oracle's float64).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bits
from oracle import quad as oq

pytestmark = pytest.mark.gpu
TOL = 1e-3


def dev_t(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def correlated(rng, shape, n=4):
    base = rng.normal(0, 0.02, size=shape)
    out = []
    for _ in range(n):
        w = base + rng.normal(0, 0.002, size=shape)
        flat = w.reshape(-1)
        idx = rng.choice(flat.size, size=max(1, flat.size // 1000), replace=False)
        flat[idx] *= 20
        out.append(w.astype(np.float16))
    return out


def packed_case(rng, K, N):
    from oracle.quad import pack_quad_layer
    ws = correlated(rng, (K, N))
    codes, luts, scales = pack_quad_layer(*ws)
    return codes, luts, scales


def run(a, codes_t, luts, scales, dev):
    from polar_pack_b200.quad_kernels import quad_bitpacked
    outs = quad_bitpacked(a, codes_t, [dev_t(t, dev) for t in luts], scales)
    torch.cuda.synchronize(dev)
    return [o.cpu().numpy() for o in outs]


@pytest.mark.parametrize("tag", ["a", "b", "c"])
@pytest.mark.parametrize("M", [1, 5])
def test_golden_reference_kernel_outputs(cuda, quad_golden, tag, M):
    g = quad_golden
    codes = g[f"{tag}_codes"]
    luts = [g[f"{tag}_lut{i}"] for i in range(7)]
    scales = list(g[f"{tag}_scales"])
    a = g[f"{tag}_a{M}"]
    outs = run(dev_t(a, cuda), dev_t(codes, cuda), luts, scales, cuda)
    ref = oq.quad_gemm(a, codes, luts, scales)
    for k in range(4):
        assert oq.rel_err(outs[k], g[f"{tag}_out{M}_{k}"]) <= TOL
        assert oq.rel_err(outs[k], ref[k]) <= TOL


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_decode_bit_exact(cuda, quad_golden, tag):
    from polar_pack_b200.quad_kernels import quad_decode
    g = quad_golden
    codes = g[f"{tag}_codes"]
    luts = [g[f"{tag}_lut{i}"] for i in range(7)]
    dec = quad_decode(dev_t(codes, cuda), [dev_t(t, cuda) for t in luts])
    ref = oq.decode_quad_fp16(codes, luts)
    for k in range(4):
        np.testing.assert_array_equal(bits(dec[k].cpu().numpy()), bits(ref[k]))


def test_decode_every_code_byte(cuda):
    """All 2^32 codes share 4 byte tables: sweep each byte through 0..255."""
    from polar_pack_b200.quad_kernels import quad_decode
    rng = np.random.default_rng(7)
    luts = [rng.normal(0, 1, 256).astype(np.float16) for _ in range(7)]
    codes = rng.integers(0, 2 ** 32, size=(256, 256), dtype=np.uint64).astype(np.uint32)
    for b in range(4):
        codes[b * 64:(b + 1) * 64] = (codes[b * 64:(b + 1) * 64] & ~np.uint32(0xFF << (8 * b))) | \
            (np.arange(256, dtype=np.uint32)[None, :] << np.uint32(8 * b))
    dec = quad_decode(dev_t(codes, cuda), [dev_t(t, cuda) for t in luts])
    ref = oq.decode_quad_fp16(codes, luts)
    for k in range(4):
        np.testing.assert_array_equal(bits(dec[k].cpu().numpy()), bits(ref[k]))


def test_decode_scaled(cuda, quad_golden):
    from polar_pack_b200.quad_kernels import quad_decode
    g = quad_golden
    codes, luts, scales = g["a_codes"], [g[f"a_lut{i}"] for i in range(7)], list(g["a_scales"])
    dec = quad_decode(dev_t(codes, cuda), [dev_t(t, cuda) for t in luts], scales)
    ref = oq.decode_quad_fp16(codes, luts)
    for k in range(4):
        want = (ref[k].astype(np.float32) * np.float32(scales[k])).astype(np.float16)
        np.testing.assert_array_equal(bits(dec[k].cpu().numpy()), bits(want))


SHAPES = [  # (M, K, N)
    (1, 64, 96), (1, 2048, 256), (2, 128, 512), (3, 37, 53), (4, 100, 36), (8, 256, 128),
    (9, 64, 64), (16, 512, 96), (17, 96, 40), (33, 64, 32), (1, 3000, 8), (5, 16, 4096),
]


@pytest.mark.parametrize("M,K,N", SHAPES)
@pytest.mark.parametrize("layout", ["kn", "nk", "strided"])
def test_random_shapes_layouts(cuda, M, K, N, layout):
    rng = np.random.default_rng(M * 1000003 + K * 101 + N)
    codes, luts, scales = packed_case(rng, K, N)
    a = rng.normal(0, 1, size=(M, K)).astype(np.float16)
    if layout == "kn":
        codes_t = dev_t(codes, cuda)
    elif layout == "nk":  # (K, N) view of an (N, K) row-major buffer
        codes_t = dev_t(codes.T.copy(), cuda).t()
    else:  # every other column of a wider buffer: no contiguous dimension
        wide = np.zeros((K, 2 * N), dtype=np.uint32)
        wide[:, ::2] = codes
        codes_t = dev_t(wide, cuda)[:, ::2]
    outs = run(dev_t(a, cuda), codes_t, luts, scales, cuda)
    ref = oq.quad_gemm(a, codes, luts, scales)
    for k in range(4):
        assert outs[k].shape == (M, N)
        assert oq.rel_err(outs[k], ref[k]) <= TOL, (k, oq.rel_err(outs[k], ref[k]))


def test_strided_activations_and_outputs(cuda):
    rng = np.random.default_rng(11)
    M, K, N = 6, 192, 160
    codes, luts, scales = packed_case(rng, K, N)
    a_big = rng.normal(0, 1, size=(M, 2 * K)).astype(np.float16)
    a_view = dev_t(a_big, cuda)[:, 1::2]  # non-unit stride along K
    outs = run(a_view, dev_t(codes, cuda), luts, scales, cuda)
    ref = oq.quad_gemm(a_big[:, 1::2], codes, luts, scales)
    for k in range(4):
        assert oq.rel_err(outs[k], ref[k]) <= TOL


def test_empty_and_k0(cuda):
    from polar_pack_b200.quad_kernels import quad_bitpacked, quad_luts
    luts = [t.to(cuda) for t in quad_luts(3.0)]
    outs = quad_bitpacked(torch.zeros((0, 8), dtype=torch.float16, device=cuda),
                          torch.zeros((8, 16), dtype=torch.uint32, device=cuda), luts, [1.0] * 4)
    assert all(o.shape == (0, 16) for o in outs)
    outs = quad_bitpacked(torch.zeros((3, 0), dtype=torch.float16, device=cuda),
                          torch.zeros((0, 16), dtype=torch.uint32, device=cuda), luts, [1.0] * 4)
    assert all(o.shape == (3, 16) and float(o.abs().max()) == 0.0 for o in outs)


def test_k_mismatch_raises_assertion(cuda):
    from polar_pack_b200.quad_kernels import quad_bitpacked, quad_luts
    luts = [t.to(cuda) for t in quad_luts(3.0)]
    with pytest.raises(AssertionError):
        quad_bitpacked(torch.zeros((1, 8), dtype=torch.float16, device=cuda),
                       torch.zeros((9, 16), dtype=torch.uint32, device=cuda), luts, [1.0] * 4)


def test_cpu_tensors_rejected():
    from polar_pack_b200.quad_kernels import quad_bitpacked, quad_luts
    with pytest.raises(RuntimeError):
        quad_bitpacked(torch.zeros((1, 8), dtype=torch.float16),
                       torch.zeros((8, 16), dtype=torch.uint32), quad_luts(3.0), [1.0] * 4)


def test_deterministic(cuda):
    rng = np.random.default_rng(5)
    codes, luts, scales = packed_case(rng, 4096, 512)
    a = dev_t(rng.normal(0, 1, (1, 4096)).astype(np.float16), cuda)
    o1 = run(a, dev_t(codes, cuda), luts, scales, cuda)
    o2 = run(a, dev_t(codes, cuda), luts, scales, cuda)
    for k in range(4):
        np.testing.assert_array_equal(bits(o1[k]), bits(o2[k]))


@pytest.mark.parametrize("K,N", [(2048, 2048), (2048, 11008), (11008, 2048), (2048, 256)])
def test_full_size_shapes(cuda, K, N):
    """BASELINE single-layer shapes, batch 1 and 4, both fast layouts.

    Reference: the numpy oracle's FP16 decode of every code
    (quad_kernels.py:103-121) followed by a float64 matmul; the GPU decode
    must equal it bit for bit on every code.
    """
    from polar_pack_b200.quad_kernels import pack_quad_layer, quad_bitpacked, quad_decode
    g = torch.Generator(device="cpu").manual_seed(K * 7 + N)
    base = torch.randn(K, N, generator=g) * 0.02
    ws = [(base + torch.randn(K, N, generator=g) * 0.002).half().to(cuda) for _ in range(4)]
    codes, luts, scales = pack_quad_layer(*ws)
    ref_dec = oq.decode_quad_fp16(codes.cpu().numpy(), [t.cpu().numpy() for t in luts])
    dec = quad_decode(codes, luts)
    for k in range(4):
        np.testing.assert_array_equal(bits(dec[k].cpu().numpy()), bits(ref_dec[k]))
    del dec
    w64 = [r.astype(np.float64) for r in ref_dec]
    for M in (1, 4):
        a = torch.randn(M, K, generator=g).half()
        a64 = a.numpy().astype(np.float64)
        for codes_v in (codes, codes.t().contiguous().t()):
            outs = quad_bitpacked(a.to(cuda), codes_v, luts, scales)
            for k in range(4):
                y_ref = (a64 @ w64[k]) * scales[k]
                err = oq.rel_err(outs[k].cpu().numpy(), y_ref)
                assert err <= TOL, (M, k, err)
