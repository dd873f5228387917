"""``GraphedStep``: a group of packed Linears replayed from one CUDA graph
together with its host copies must give the eager group's result bit for
bit (same kernels, deterministic reductions), for new host inputs on every
call, and must refuse unpinned host inputs.
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = [(256, 512), (2048, 256), (8, 64), (1000, 1028)]  # (N out, K in)


def _layers(dev):
    from polar_pack_b200.quadpack import DevicePackedStream, pack_quad_device
    n = sum(N * K for N, K in SHAPES)
    g = torch.Generator(device=dev)
    g.manual_seed(9)
    base = torch.randn(n, generator=g, device=dev) * 0.02
    models = [(base + torch.randn(n, generator=g, device=dev) * 0.002).half() for _ in range(4)]
    st = DevicePackedStream(pack_quad_device(models, plug_cap=0.05, seed=42, windows=8, window=65536))
    layers, off = [], 0
    for N, K in SHAPES:
        layers.append(st.linear(off, N, K))
        off += N * K
    return layers


def test_graphed_step_matches_eager(cuda):
    from polar_pack_b200.parallel import GraphedStep, RowShardedGroup
    from polar_pack_b200.quadpack import quad_linear
    layers = _layers(cuda)
    Ns = [N for N, _ in SHAPES]
    grp = RowShardedGroup([lambda x, out, l=l: quad_linear(x, l, out=out) for l in layers], Ns, writes_out=True)
    sizes = [K for _, K in SHAPES]
    hx = torch.empty(sum(sizes), dtype=torch.float16).pin_memory()
    dxf = torch.empty_like(hx, device=cuda)
    dx, o = [], 0
    for K in sizes:
        dx.append(dxf[o:o + K].view(1, K))
        o += K
    step = GraphedStep(lambda: (grp(dx), grp.raw())[1], hx, dxf, torch.cuda.Stream(cuda))
    gen = torch.Generator().manual_seed(4)
    for _ in range(3):
        hx.copy_(torch.randn(hx.shape, generator=gen).half())
        got = step()
        torch.cuda.synchronize(cuda)
        got = got.clone()
        dxf.copy_(hx)
        grp(dx)
        ref = grp.raw().cpu()
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
        assert got.abs().sum() > 0


def test_graphed_step_needs_pinned_input(cuda):
    from polar_pack_b200.parallel import GraphedStep
    with pytest.raises(ValueError):
        GraphedStep(lambda: torch.zeros(1, device=cuda), torch.zeros(4), torch.zeros(4, device=cuda),
                    torch.cuda.Stream(cuda))
