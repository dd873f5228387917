"""Launch overlap (programmatic dependent launch) keeps results unchanged.

With ``pp_set_launch_overlap(1)`` each quad kernel may start while the
previous kernel of its stream runs, and waits for it before touching
activations, the workspace or outputs.  A chain of dependent Linears (each
consuming the previous one's output) run back to back without host syncs
must give bit-identical results with overlap on and off.
"""
import numpy as np
import pytest
import torch

from conftest import bits
from oracle import formats as of

pytestmark = pytest.mark.gpu

# (out, in): each layer's input width is the previous layer's output width
CHAIN = [(512, 256), (256, 512), (1024, 256), (256, 1024), (64, 256)]


@pytest.fixture(scope="module")
def chain_pack(cuda):
    from polar_pack_b200.quadpack import QuadPackDevice, QuadPackFile
    rng = np.random.default_rng(77)
    n = sum(o * i for o, i in CHAIN)
    base = rng.normal(0, 0.02, size=n)
    models = []
    for _ in range(4):
        w = base + rng.normal(0, 0.002, size=n)
        idx = rng.choice(n, size=n // 1000, replace=False)
        w[idx] *= 20
        models.append(w.astype(np.float16).astype(np.float32))
    buf = of.pack_quad_bytes(models, plug_cap=0.05, threshold_windows=8, window=4096)
    pk = QuadPackDevice(QuadPackFile(buf), cuda)
    layers, off = [], 0
    for (N, K) in CHAIN:
        layers.append(pk.linear(off, N, K))
        off += N * K
    return layers


def _run_chain(layers, x, reps):
    outs = []
    y = x
    for _ in range(reps):
        y = x
        for lin in layers:
            ys = lin(y)
            y = ys[(len(outs) + lin.N) % 4]    # feed one of the four models onward
        outs.append(y)
    torch.cuda.synchronize()
    return [o.clone() for o in outs]


def _run_gemm_chain(cuda, x, reps):
    from polar_pack_b200.quad_kernels import pack_quad_layer, quad_bitpacked
    g = torch.Generator(device="cpu").manual_seed(3)
    mats = []
    for (N, K) in CHAIN:
        ws = [(torch.randn(K, N, generator=g) * 0.02).half().to(cuda) for _ in range(4)]
        mats.append(pack_quad_layer(*ws))
    res = []
    for _ in range(reps):
        y = x
        for (codes, luts, scales) in mats:
            y = quad_bitpacked(y, codes, luts, scales)[1]
        res.append(y)
    torch.cuda.synchronize()
    return [r.clone() for r in res]


def test_overlap_gives_identical_results(cuda, chain_pack):
    from polar_pack_b200 import _lib
    x = torch.randn(3, CHAIN[0][1], generator=torch.Generator().manual_seed(1)).half().to(cuda)
    prev = _lib.set_launch_overlap(False)
    try:
        ref = _run_chain(chain_pack, x, 4)
        ref_g = _run_gemm_chain(cuda, x, 3)
        _lib.set_launch_overlap(True)
        got = _run_chain(chain_pack, x, 4)
        got_g = _run_gemm_chain(cuda, x, 3)
    finally:
        _lib.set_launch_overlap(prev)
    for a, b in zip(ref + ref_g, got + got_g):
        assert torch.isfinite(a.float()).all()
        np.testing.assert_array_equal(bits(a.cpu().numpy()), bits(b.cpu().numpy()))
