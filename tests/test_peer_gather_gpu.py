"""Outputs gathered through peer memory (pp_quad_linear_gather, pp_gather_wait).

On one GPU: a gathered Linear stores into its own buffer, which must equal
the ordinary fused call bit for bit (same kernel, same partition), the
epoch must count the launches, and a wait on a flag that nothing sets must
give up with status 3 after its bounded number of polls.  On two GPUs (child
processes over NCCL on 127.0.0.1): every rank's gathered result must equal
the full Linear computed on one GPU.
"""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import quad as oq

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
TOL = 1e-3


def _stream(dev, shapes, seed=5):
    """A synthetic packed stream holding the given (N, K) Linears in order."""
    sys.path.insert(0, str(ROOT))
    from polar_pack_b200.quadpack import DevicePackedStream, pack_quad_device
    n = sum(N * K for N, K in shapes)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    base = torch.randn(n, generator=g, device=dev) * 0.02
    models = []
    for _ in range(4):
        w = base + torch.randn(n, generator=g, device=dev) * 0.002
        idx = torch.randint(0, n, (max(1, n // 1000),), generator=g, device=dev)
        w[idx] *= 20
        models.append(w.half())
    p = pack_quad_device(models, plug_cap=0.05, seed=42, windows=8, window=65536)
    return DevicePackedStream(p)


SHAPES = [(256, 512), (2048, 256), (8, 64), (1000, 1028)]  # (N out, K in)
# rows not a multiple of 8: the first launch mixes 16-byte tile stores with a
# 2-byte tail tile, the second starts at row 1001 (2-byte stores throughout),
# the third at the aligned row 1008 again
RAGGED = [(1001, 512), (7, 64), (256, 128)]


@pytest.mark.parametrize("SHAPES", [SHAPES, RAGGED], ids=["aligned", "ragged"])
def test_gather_single_rank_matches_fused(cuda, SHAPES):
    from polar_pack_b200.parallel import PeerBuffers, PeerShardedGroup
    from polar_pack_b200.quadpack import quad_linear
    st = _stream(cuda, SHAPES)
    layers, off = [], 0
    for N, K in SHAPES:
        layers.append(st.linear(off, N, K))
        off += N * K
    Ns = [N for N, _ in SHAPES]
    peers = PeerBuffers(4 * sum(Ns), nbuf=2, device=cuda)
    grp = PeerShardedGroup(layers, Ns, [0] * len(Ns), peers)
    g = torch.Generator(device=cuda)
    g.manual_seed(3)
    xs = [torch.randn(1, K, generator=g, device=cuda).half() for _, K in SHAPES]
    ref = [quad_linear(x, l) for x, l in zip(xs, layers)]
    first = None
    for call in range(3):
        b = call % 2
        y = grp(xs, b).clone()
        torch.cuda.synchronize(cuda)
        col = 0
        for (N, _), r in zip(SHAPES, ref):
            for k in range(4):
                if grp.single_launch:   # one grouped launch: each Linear on its SM share (own split-K order)
                    assert oq.rel_err(y[k, col:col + N].float().cpu().numpy(),
                                      r[k][0].float().cpu().numpy()) <= TOL, (N, k)
                else:                   # one launch per Linear: the same kernel and partition as the plain call
                    assert torch.equal(y[k, col:col + N].view(torch.int16), r[k][0].view(torch.int16)), (N, k)
            col += N
        if first is None:
            first = y
        else:
            assert torch.equal(y.view(torch.int16), first.view(torch.int16))   # deterministic
    ep = peers.mem[peers.epoch_off:peers.epoch_off + 8].view(torch.int32).cpu().tolist()
    per_call = 1 if grp.single_launch else len(SHAPES)   # epochs: launches made into buffers 0 and 1
    assert ep == [2 * per_call, per_call]
    assert int(peers.status.item()) == 0
    peers.close()


def test_gather_wait_gives_up(cuda):
    """Rank 1 of a pretended world of 2 never publishes: the wait must end
    by itself with status 3 (no hang; the context stays usable)."""
    from polar_pack_b200 import _lib
    from polar_pack_b200.parallel import PeerBuffers
    peers = PeerBuffers(1024, nbuf=1, device=cuda)
    peers.mem[peers.epoch_off:peers.epoch_off + 4].view(torch.int32).fill_(1)   # expect epoch 1
    peers.mem[peers.flags_off:peers.flags_off + 4].view(torch.int32).fill_(1)   # rank 0 published
    # world 2: the second flag word lies in the zero padding of the flag region
    _lib.call("pp_gather_wait", peers.local_flags(0), 2, peers.epoch_ptr(0), peers.status.data_ptr(),
              torch.cuda.current_stream(cuda).cuda_stream)
    torch.cuda.synchronize(cuda)
    assert int(peers.status.item()) == 3
    x = torch.ones(4, device=cuda)
    assert float((x * 2).sum().item()) == 8.0   # the context still works
    peers.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        import torch.distributed as dist
        from datetime import timedelta
        sys.path.insert(0, str(ROOT))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
        from polar_pack_b200.parallel import PeerBuffers, PeerShardedGroup, row_shard
        from polar_pack_b200.quadpack import quad_linear
        st = _stream(dev, SHAPES)
        shards, full, r0s, off = [], [], [], 0
        for N, K in SHAPES:
            n0, n1 = row_shard(N, world, rank)
            shards.append(st.linear(off + n0 * K, n1 - n0, K))
            full.append(st.linear(off, N, K))
            r0s.append(n0)
            off += N * K
        Ns = [N for N, _ in SHAPES]
        peers = PeerBuffers(4 * sum(Ns), nbuf=2, device=dev)
        grp = PeerShardedGroup(shards, Ns, r0s, peers)
        g = torch.Generator(device=dev)
        g.manual_seed(3)
        xs = [torch.randn(1, K, generator=g, device=dev).half() for _, K in SHAPES]
        ok = True
        for call in range(4):
            y = grp(xs, call % 2).float().cpu().numpy()
            col = 0
            for (N, _), l, x in zip(SHAPES, full, xs):
                r = quad_linear(x, l)
                for k in range(4):
                    ok &= oq.rel_err(y[k, col:col + N], r[k][0].float().cpu().numpy()) <= TOL
                col += N
        ok &= int(peers.status.item()) == 0
        peers.close()
        dist.destroy_process_group()
        q.put((rank, bool(ok), ""))
    except Exception as e:
        q.put((rank, False, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_gather_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in res), res
