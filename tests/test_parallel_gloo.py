"""Row-sharded Linear host logic on 2 CPU ranks (gloo): shard bounds, padded
all-gather, reassembly -- and a rank that never joins fails the others on the
host within the process-group timeout instead of hanging."""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))


def _worker_gather(rank, world, port, N, K, M, q):
    try:
        _gather_body(rank, world, port, N, K, M, q)
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, False, repr(e)))


def _gather_body(rank, world, port, N, K, M, q):
    sys.path.insert(0, str(ROOT))
    from oracle import quad as oq
    from polar_pack_b200.parallel import RowShardedLinear, row_shard
    _init(rank, world, port)
    rng = np.random.default_rng(0)   # same weights on every rank
    ws = [rng.normal(0, 0.02, (N, K)).astype(np.float16) for _ in range(4)]
    x = rng.normal(0, 1, (M, K)).astype(np.float16)
    n0, n1 = row_shard(N, world, rank)

    def local_fn(xt):
        return [torch.from_numpy((xt.numpy().astype(np.float64) @ w[n0:n1].T.astype(np.float64))
                                 .astype(np.float16)) for w in ws]

    lin = RowShardedLinear(local_fn, N)
    outs = lin(torch.from_numpy(x))
    full = [(x.astype(np.float64) @ w.T.astype(np.float64)).astype(np.float16) for w in ws]
    ok = all(np.array_equal(o.numpy(), f) for o, f in zip(outs, full))
    q.put((rank, ok, [tuple(o.shape) for o in outs]))
    dist.destroy_process_group()


@pytest.mark.parametrize("N", [16, 13])
def test_row_sharded_gather_matches_full(N):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, K, M = 2, 24, 3
    port = free_port()
    procs = [ctx.Process(target=_worker_gather, args=(r, world, port, N, K, M, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok, _ in res)
    assert all(shapes == [(M, N)] * 4 for _, _, shapes in res)


def _worker_group(rank, world, port, Ns, K, M, q, writes_out=False):
    try:
        sys.path.insert(0, str(ROOT))
        from polar_pack_b200.parallel import RowShardedGroup, row_shard
        _init(rank, world, port)
        rng = np.random.default_rng(1)
        wss = [[rng.normal(0, 0.02, (N, K)).astype(np.float16) for _ in range(4)] for N in Ns]
        xs = [rng.normal(0, 1, (M, K)).astype(np.float16) for _ in Ns]

        def make(ws, N):
            n0, n1 = row_shard(N, world, rank)
            fn = lambda xt: [torch.from_numpy((xt.numpy().astype(np.float64) @ w[n0:n1].T.astype(np.float64))
                                              .astype(np.float16)) for w in ws]
            if not writes_out:
                return fn

            def into(xt, out):  # writes into the group's send-buffer views
                for dst, src in zip(out, fn(xt)):
                    dst.copy_(src)
            return into

        grp = RowShardedGroup([make(ws, N) for ws, N in zip(wss, Ns)], Ns, writes_out=writes_out)
        outs = grp([torch.from_numpy(x) for x in xs])
        outs = grp([torch.from_numpy(x) for x in xs])  # buffers are reused: a second call gives the same
        ok = True
        for o, ws, x in zip(outs, wss, xs):
            full = [(x.astype(np.float64) @ w.T.astype(np.float64)).astype(np.float16) for w in ws]
            ok &= all(np.array_equal(a.numpy(), f) for a, f in zip(o, full))
        q.put((rank, ok, [tuple(t.shape) for o in outs for t in o]))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, False, repr(e)))


@pytest.mark.parametrize("writes_out", [False, True])
def test_grouped_gather_matches_full(writes_out):
    """Several Linears of different widths (one not divisible by the world
    size) gathered by one collective, with local functions that return
    their outputs or write them into the send buffer."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, K, M, Ns = 2, 20, 2, [16, 13, 6]
    port = free_port()
    procs = [ctx.Process(target=_worker_group, args=(r, world, port, Ns, K, M, q, writes_out))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok, _ in res), res
    assert all(shapes == [(M, N) for N in Ns for _ in range(4)] for _, _, shapes in res)


def test_row_shard_bounds():
    from polar_pack_b200.parallel import row_shard, shard_width
    for N in (1, 7, 8, 16, 63, 64, 256, 2048, 11008, 151936):
        for world in (1, 2, 4, 8):
            b = [row_shard(N, world, r) for r in range(world)]
            assert b[0][0] == 0 and b[-1][1] == N
            assert all(b[i][1] == b[i + 1][0] for i in range(world - 1))
            assert max(n1 - n0 for n0, n1 in b) <= shard_width(N, world)
            if N >= 8 * world:
                assert all(n0 % 8 == 0 for n0, _ in b)        # whole 8-row output tiles
                assert min(n1 - n0 for n0, n1 in b) >= 8
                assert max(n1 - n0 for n0, n1 in b) - min(n1 - n0 for n0, n1 in b) <= 8
            else:
                assert max(n1 - n0 for n0, n1 in b) - min(n1 - n0 for n0, n1 in b) <= 1
    with pytest.raises(ValueError):
        row_shard(8, 2, 2)


def _worker_missing_peer(rank, world, port, q):
    sys.path.insert(0, str(ROOT))
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        dist.barrier()
        _put_and_flush(q, (rank, "left"))
        os._exit(0)          # leaves between steps, never joins the next collective
    dist.barrier()
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        _put_and_flush(q, (rank, "no error"))
    except Exception as e:  # timeout or peer-closed error, surfaced on the host
        _put_and_flush(q, (rank, f"error: {type(e).__name__}"))
    os._exit(0)


def _put_and_flush(q, item):
    q.put(item)
    q.close()
    q.join_thread()


def test_missing_rank_fails_on_host_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker_missing_peer, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res[1] == "left"
    assert res[0].startswith("error")


def test_grouped_single_rank_views():
    """One rank: the outputs are views of the reused send buffer."""
    from polar_pack_b200.parallel import RowShardedGroup
    Ns, M = [5, 3], 2

    def fn(v):
        return lambda x, out: [o.fill_(v + k) for k, o in enumerate(out)]
    grp = RowShardedGroup([fn(10), fn(20)], Ns, writes_out=True)
    outs = grp([torch.zeros(M, 4), torch.zeros(M, 4)])
    raw = grp.raw()
    assert raw.shape == (4, M, sum(Ns))
    assert [tuple(o.shape) for o in outs[0]] == [(M, 5)] * 4 and [tuple(o.shape) for o in outs[1]] == [(M, 3)] * 4
    assert float(raw[2, 0, 0]) == 12 and float(raw[3, 1, 6]) == 23
    assert outs[1][0].data_ptr() == raw[0, :, 5:].data_ptr()
