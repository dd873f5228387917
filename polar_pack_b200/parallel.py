"""Row-sharded (column-parallel) packed Linears across the GPUs of one node.

Output features of a Linear are independent, and in the file layout each
Linear is ``(out, in)`` row-major, so the rows ``[n0, n1)`` owned by one rank
are one contiguous slice of the code stream (and of the sorted plug table).
Each rank streams only its slice; the four models' FP16 outputs are then
all-gathered (NCCL over NVLink on GPUs, gloo in the CPU tests).  There is no
cross-rank reduction.

The reference runs one model per process on one GPU; this module is new
(north_star item 3).
"""
from __future__ import annotations

from typing import Callable, Sequence

import torch
import torch.distributed as dist


def row_shard(N: int, world: int, rank: int) -> tuple[int, int]:
    """Rows ``[n0, n1)`` of rank ``rank``: contiguous, sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    return N * rank // world, N * (rank + 1) // world


def shard_width(N: int, world: int) -> int:
    """Padded per-rank width used for the all-gather (equal sizes on every rank)."""
    return -(-N // world)


class RowShardedLinear:
    """Runs ``local_fn`` on this rank's rows and all-gathers the outputs.

    ``local_fn(x) -> list of n_out tensors (M, n1 - n0)`` computes the local
    row shard (on a GPU: one fused kernel launch).  ``__call__`` returns
    ``n_out`` full ``(M, N)`` tensors.  Every rank must call it with the same
    ``M`` in the same order (one collective per call).
    """

    def __init__(self, local_fn: Callable[[torch.Tensor], Sequence[torch.Tensor]], N: int,
                 group=None, n_out: int = 4):
        self.local_fn = local_fn
        self.N = N
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.n0, self.n1 = row_shard(N, self.world, self.rank)
        self.width = shard_width(N, self.world)
        self.n_out = n_out

    def __call__(self, x: torch.Tensor) -> list[torch.Tensor]:
        M = x.shape[0]
        local = self.local_fn(x)
        if self.world == 1:
            return list(local)
        n_loc = self.n1 - self.n0
        send = torch.zeros((self.n_out, M, self.width), dtype=local[0].dtype, device=local[0].device)
        for k in range(self.n_out):
            send[k, :, :n_loc] = local[k]
        # concatenated along dim 0 (the form both NCCL and gloo accept)
        recv = torch.empty((self.world * self.n_out, M, self.width), dtype=send.dtype, device=send.device)
        dist.all_gather_into_tensor(recv, send, group=self.group)
        recv = recv.view(self.world, self.n_out, M, self.width)
        outs = []
        for k in range(self.n_out):
            parts = []
            for r in range(self.world):
                a, b = row_shard(self.N, self.world, r)
                parts.append(recv[r, k, :, :b - a])
            outs.append(torch.cat(parts, dim=1))
        return outs


class RowShardedGroup:
    """Several independent row-sharded Linears with ONE all-gather.

    For Linears that do not feed each other (q/k/v, gate/up, or the
    benchmark's sweep), every rank computes its row shard of each into one
    send buffer of ``n_out`` blocks ``(M, sum of shard widths)`` and a single
    collective gathers everything.  ``__call__(xs)`` returns, per Linear,
    ``n_out`` full ``(M, N_j)`` tensors; one collective instead of one per
    Linear.

    ``writes_out=True`` means ``local_fns[j](x, out)`` writes its outputs
    into ``out`` (``n_out`` strided ``(M, rows of this rank)`` views of the
    send buffer, as ``quad_linear(x, layer, out=...)`` accepts); otherwise
    ``local_fns[j](x)`` returns them and they are copied in.  The send and
    receive buffers are kept per batch size and reused: on one GPU the
    returned tensors are views of the send buffer, and ``raw()`` is the last
    call's buffer (``(n_out, M, total)`` on one GPU, ``(world * n_out, M,
    total)`` gathered, rank-major) for callers that read the result once,
    e.g. a single device-to-host copy.
    """

    def __init__(self, local_fns: Sequence[Callable], Ns: Sequence[int], group=None, n_out: int = 4,
                 writes_out: bool = False):
        if len(local_fns) != len(Ns):
            raise ValueError("one local function per Linear")
        self.local_fns = list(local_fns)
        self.Ns = list(Ns)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.widths = [shard_width(N, self.world) for N in self.Ns]
        self.n_out = n_out
        self.writes_out = writes_out
        self._bufs: dict = {}
        self._last = None

    def _buffers(self, M, dev, dt):
        key = (M, dev, dt)
        b = self._bufs.get(key)
        if b is None:
            total = sum(self.widths)
            # zero-filled once: the padding columns of short shards stay zero
            send = torch.zeros((self.n_out, M, total), dtype=dt, device=dev)
            recv = torch.empty((self.world * self.n_out, M, total), dtype=dt, device=dev) \
                if self.world > 1 else None
            outs, col = [], 0
            for N, w in zip(self.Ns, self.widths):
                a, b_ = row_shard(N, self.world, self.rank)
                outs.append([send[k, :, col:col + b_ - a] for k in range(self.n_out)])
                col += w
            b = self._bufs[key] = (send, recv, outs)
        return b

    def raw(self) -> torch.Tensor:
        return self._last

    def __call__(self, xs: Sequence[torch.Tensor], dtype=torch.float16) -> list[list[torch.Tensor]]:
        M = xs[0].shape[0]
        send, recv, outs = self._buffers(M, xs[0].device, dtype)
        for fn, x, out in zip(self.local_fns, xs, outs):
            if self.writes_out:
                fn(x, out)
            else:
                for dst, src in zip(out, fn(x)):
                    dst.copy_(src)
        if self.world == 1:
            self._last = send
            return [list(o) for o in outs]
        dist.all_gather_into_tensor(recv, send, group=self.group)
        self._last = recv
        rv = recv.view(self.world, self.n_out, M, -1)
        res, col = [], 0
        for N, w in zip(self.Ns, self.widths):
            outs_j = []
            for k in range(self.n_out):
                parts = []
                for r in range(self.world):
                    a, b = row_shard(N, self.world, r)
                    parts.append(rv[r, k, :, col:col + b - a])
                outs_j.append(torch.cat(parts, dim=1))
            res.append(outs_j)
            col += w
        return res


def shard_quad_linear(pack, offset: int, N: int, K: int, world: int, rank: int):
    """This rank's row slice of the packed Linear at flat ``offset`` (file layout)."""
    n0, n1 = row_shard(N, world, rank)
    return pack.linear(offset + n0 * K, n1 - n0, K)
