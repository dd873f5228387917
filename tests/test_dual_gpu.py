"""GPU parity of the dual kernel (drop-in ``polar_dual_bitpacked``)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bits
from oracle import dual as od
from oracle.quad import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-3


def dev_t(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def dual_args(g, tag, dev):
    return [dev_t(g[f"{tag}_{n}"], dev) for n in ("bmax", "amp_lut", "cos_lut", "sin_lut")]


@pytest.mark.parametrize("tag", ["a", "b"])
@pytest.mark.parametrize("M", [1, 4])
def test_golden_reference_kernel_outputs(cuda, dual_golden, tag, M):
    from polar_pack_b200.polar_kernels import polar_dual_bitpacked
    g = dual_golden
    o = polar_dual_bitpacked(dev_t(g[f"{tag}_a{M}"], cuda), dev_t(g[f"{tag}_packed"], cuda),
                             *dual_args(g, tag, cuda))
    ref = od.dual_gemm(g[f"{tag}_a{M}"], g[f"{tag}_packed"],
                       *[g[f"{tag}_{n}"] for n in ("bmax", "amp_lut", "cos_lut", "sin_lut")])
    for j in range(2):
        y = o[j].cpu().numpy()
        assert rel_err(y, g[f"{tag}_out{M}_{j}"]) <= TOL
        assert rel_err(y, ref[j]) <= TOL


@pytest.mark.parametrize("tag", ["a", "b"])
def test_decode_bit_exact(cuda, dual_golden, tag):
    from polar_pack_b200.polar_kernels import dual_decode
    g = dual_golden
    b = dual_decode(dev_t(g[f"{tag}_packed"], cuda), *dual_args(g, tag, cuda))
    ref = od.decode_dual_fp16(g[f"{tag}_packed"], *[g[f"{tag}_{n}"] for n in ("bmax", "amp_lut", "cos_lut", "sin_lut")])
    for j in range(2):
        np.testing.assert_array_equal(bits(b[j].cpu().numpy()), bits(ref[j]))


# batch 1 with N % 256 == 0 (and the default group of 32) runs on the TMA
# engine (dual_tma.cu), ragged K included; the rest on the register engine
SHAPES = [(1, 64, 96), (1, 2048, 256), (3, 37, 56), (4, 100, 64), (8, 256, 128), (9, 64, 64),
          (16, 512, 192), (17, 96, 40), (2, 33, 7), (1, 4096, 512), (1, 100, 256), (1, 37, 768),
          (1, 1000, 1024)]


@pytest.mark.parametrize("M,K,N", SHAPES)
@pytest.mark.parametrize("layout", ["kn", "strided"])
def test_random_shapes(cuda, M, K, N, layout):
    from polar_pack_b200.polar_kernels import polar_dual_bitpacked
    rng = np.random.default_rng(M * 7919 + K * 31 + N)
    base = rng.normal(0, 0.02, size=(K, N))
    w1 = (base + rng.normal(0, 0.002, size=(K, N))).astype(np.float32)
    w2 = (base + rng.normal(0, 0.002, size=(K, N))).astype(np.float32)
    packed, bmax, amp_lut, cos_lut, sin_lut = od.quantize_polar_bitpacked(w1, w2)
    a = rng.normal(0, 1, size=(M, K)).astype(np.float16)
    if layout == "kn":
        p_t = dev_t(packed, cuda)
    else:
        wide = np.zeros((K, 2 * N), dtype=np.int16)
        wide[:, ::2] = packed
        p_t = dev_t(wide, cuda)[:, ::2]
    o = polar_dual_bitpacked(dev_t(a, cuda), p_t, dev_t(bmax, cuda), dev_t(amp_lut, cuda),
                             dev_t(cos_lut, cuda), dev_t(sin_lut, cuda))
    ref = od.dual_gemm(a, packed, bmax, amp_lut, cos_lut, sin_lut)
    for j in range(2):
        assert rel_err(o[j].cpu().numpy(), ref[j]) <= TOL


def test_k_mismatch_raises_assertion(cuda):
    from polar_pack_b200.polar_kernels import dual_luts, polar_dual_bitpacked
    amp, c, s = dual_luts(device=cuda)
    with pytest.raises(AssertionError):
        polar_dual_bitpacked(torch.zeros((1, 8), dtype=torch.float16, device=cuda),
                             torch.zeros((9, 16), dtype=torch.int16, device=cuda),
                             torch.ones(8, dtype=torch.float16, device=cuda), amp, c, s)


@pytest.mark.parametrize("K,N", [(2048, 2048), (2048, 11008), (11008, 2048)])
def test_full_size(cuda, K, N):
    from polar_pack_b200.polar_kernels import dual_decode, polar_dual_bitpacked, quantize_polar_bitpacked
    g = torch.Generator(device="cpu").manual_seed(K + N)
    base = torch.randn(K, N, generator=g) * 0.02
    w1 = (base + torch.randn(K, N, generator=g) * 0.002).to(cuda)
    w2 = (base + torch.randn(K, N, generator=g) * 0.002).to(cuda)
    packed, bmax, amp_lut, cos_lut, sin_lut = quantize_polar_bitpacked(w1, w2)
    b = dual_decode(packed, bmax, amp_lut, cos_lut, sin_lut)
    a = torch.randn(1, K, generator=g).half().to(cuda)
    o = polar_dual_bitpacked(a, packed, bmax, amp_lut, cos_lut, sin_lut)
    for j in range(2):
        y_ref = a.double() @ b[j].double()
        assert float((o[j].double() - y_ref).abs().max() / y_ref.abs().max()) <= TOL
