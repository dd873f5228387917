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


SHARD_ALIGN = 8   # rows: one GEMV output tile


def _shard_bound(N: int, world: int, r: int) -> int:
    if r >= world:
        return N
    if N < SHARD_ALIGN * world:          # no empty shard for a tiny Linear: split row by row
        return N * r // world
    tiles = -(-N // SHARD_ALIGN)
    return tiles * r // world * SHARD_ALIGN


def row_shard(N: int, world: int, rank: int) -> tuple[int, int]:
    """Rows ``[n0, n1)`` of rank ``rank``: contiguous.  When every rank can
    hold 8 rows, the ranks take equal shares (within one) of the 8-row output
    tiles, so the inner boundaries lie on multiples of 8 rows: a rank's tiles
    are whole tiles of the unsharded Linear and reach the gathered buffers as
    16-byte stores (sizes differ by at most 8 rows).  A Linear of fewer than
    8 rows per rank is split row by row (sizes differ by at most one)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    return _shard_bound(N, world, rank), _shard_bound(N, world, rank + 1)


def shard_width(N: int, world: int) -> int:
    """Padded per-rank width used for the all-gather (equal sizes on every rank)."""
    return max(_shard_bound(N, world, r + 1) - _shard_bound(N, world, r) for r in range(world))


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


# ------------------------------------------------------- peer gather ----
def _align(n: int, a: int = 256) -> int:
    return -(-n // a) * a


class PeerBuffers:
    """Gather buffers that every rank of a process group can write.

    One device allocation per rank holds ``nbuf`` buffers of ``elems`` FP16
    elements (the gathered outputs, model-major), a flag array per buffer
    (``world`` u32: rank q's latest published epoch in word q) and this
    rank's epoch counters (one u32 per buffer).  Every rank maps every other
    rank's allocation through CUDA IPC (handles exchanged over the process
    group), so a kernel on this GPU can store into all of them over NVLink.
    Zero-filled once; epochs and flags only grow afterwards.
    """

    def __init__(self, elems: int, nbuf: int = 2, group=None, device=None):
        import ctypes

        from . import _lib
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > 8:
            raise ValueError("peer gather supports up to 8 ranks")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.elems, self.nbuf = elems, nbuf
        self.data_bytes = _align(elems * 2)
        self.flags_off = nbuf * self.data_bytes
        self.epoch_off = self.flags_off + _align(nbuf * self.world * 4)
        total = self.epoch_off + _align(nbuf * 4)
        self.mem = torch.zeros(total, dtype=torch.uint8, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        handle = (ctypes.c_char * 64)()
        off = _lib._size_t()
        _lib.call("pp_ipc_handle", self.mem.data_ptr(), handle, ctypes.byref(off))
        mine = (bytes(handle), int(off.value))
        allh = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(allh, mine, group=group)
        else:
            allh = [mine]
        self.bases, self._opened = [], []
        for q, (h, o) in enumerate(allh):
            if q == self.rank:
                self.bases.append(self.mem.data_ptr())
                continue
            p = ctypes.c_void_p()
            _lib.call("pp_ipc_open", ctypes.create_string_buffer(h, 64), ctypes.byref(p))
            self._opened.append(p.value)
            self.bases.append(p.value + o)
        if self.world > 1:
            dist.barrier(group=group)

    def out_ptrs(self, b: int) -> list[int]:
        """Buffer ``b`` of every rank, as mapped here."""
        return [base + b * self.data_bytes for base in self.bases]

    def flag_ptrs(self, b: int) -> list[int]:
        """This rank's flag word of buffer ``b`` in every rank's flag array."""
        return [base + self.flags_off + (b * self.world + self.rank) * 4 for base in self.bases]

    def local_flags(self, b: int) -> int:
        return self.mem.data_ptr() + self.flags_off + b * self.world * 4

    def epoch_ptr(self, b: int) -> int:
        return self.mem.data_ptr() + self.epoch_off + b * 4

    def view(self, b: int) -> torch.Tensor:
        """This rank's buffer ``b`` as FP16 elements."""
        return self.mem[b * self.data_bytes:b * self.data_bytes + self.elems * 2].view(torch.float16)

    def wait(self, b: int, stream=None) -> None:
        """Make the stream wait until every rank has published buffer ``b``."""
        from . import _lib
        s = stream if stream is not None else torch.cuda.current_stream(self.device).cuda_stream
        _lib.call("pp_gather_wait", self.local_flags(b), self.world, self.epoch_ptr(b), self.status.data_ptr(), s)

    def close(self) -> None:
        from . import _lib
        if self.world > 1:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)  # no peer still writes into a mapping about to go
        for p in self._opened:
            _lib.call("pp_ipc_close", p)
        self._opened = []


class PeerShardedGroup:
    """Row-sharded batch-1 Linears whose outputs are gathered through peer
    memory instead of an all-gather.

    ``layers[j]`` is this rank's row shard (a ``QuadLinearSlice`` with its
    unit plugs) of a Linear with ``Ns[j]`` rows; ``row0s[j]`` is the shard's
    first row.  A call launches every Linear with ``pp_quad_linear_gather``
    into buffer ``b`` (model-major: model k, Linear j, row n at
    ``k * sum(Ns) + offset_j + n``), then waits for every rank.  When every
    rank's shards allow it (``single_launch``, agreed over the process group)
    the Linears run as one grouped launch that publishes one epoch per call
    (``pp_quad_linear_group_gather``); else one launch (and epoch) per
    Linear.  The result is ``peers.view(b)`` viewed as ``(4, sum(Ns))``,
    which the next call into the same buffer overwrites: alternate the
    buffers.
    """

    def __init__(self, layers, Ns, row0s, peers: PeerBuffers):
        import ctypes

        from . import _lib
        from .quadpack import quad_linear_workspace_bytes
        self.layers, self.Ns, self.peers = list(layers), list(Ns), peers
        self.total = sum(self.Ns)
        if 4 * self.total > peers.elems:
            raise ValueError("peer buffers too small for the group")
        self.cols = [sum(self.Ns[:j]) for j in range(len(self.Ns))]
        self.row0s = list(row0s)
        dev = peers.device
        nb = max(quad_linear_workspace_bytes(1, l.N, l.K) for l in self.layers)
        self.ws = torch.zeros(max(nb, 256), dtype=torch.uint8, device=dev)
        self._lib = _lib.load()
        self._args = {}
        self._descs = {}
        # One grouped launch per call (pp_quad_linear_group_gather: one epoch
        # per call) when every rank's shards allow it; the ranks must agree,
        # since each waits for the others' epoch counts.
        from .quadpack import linear_desc
        probe = [torch.empty((1, l.K), dtype=torch.float16, device=dev) for l in self.layers]
        d = (_lib.QuadLinearDesc * len(self.layers))(*[linear_desc(x, l, None) for x, l in zip(probe, self.layers)])
        ok = bool(self._lib.pp_quad_linear_group_single_launch(len(self.layers), d))
        if peers.world > 1:
            t = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MIN, group=peers.group)
            ok = bool(t.item())
        self.single_launch = ok
        if ok:
            nb_g = _lib._size_t()
            _lib.check(self._lib.pp_quad_linear_group_workspace_bytes(len(self.layers), d, ctypes.byref(nb_g)))
            if nb_g.value > self.ws.numel():
                self.ws = torch.zeros(nb_g.value, dtype=torch.uint8, device=dev)
        for b in range(peers.nbuf):
            outs = (ctypes.c_void_p * 8)(*peers.out_ptrs(b))
            flags = (ctypes.c_void_p * 8)(*peers.flag_ptrs(b))
            row = []
            for l, c, r0 in zip(self.layers, self.cols, self.row0s):
                row.append((l.codes.data_ptr(), l.K, _lib.ptr(l.plug_idx), _lib.ptr(l.plug_vals),
                            _lib.ptr(l.plug_window_base), ctypes.c_uint32(l.offset & 0xFFFFFFFF),
                            _lib.ptr(l.unit_plugs), _lib.ptr(l.unit_plug_off), l.pack.tables.data_ptr(),
                            _lib.floats4(l.pack.scales), peers.world, outs, self.total, c + r0, flags,
                            peers.epoch_ptr(b), l.N, l.K))
            self._args[b] = (row, outs, flags)

    def _group_args(self, xs, b):
        """Descriptors and gather arguments of one grouped launch into buffer b."""
        import ctypes

        from . import _lib
        from .quadpack import linear_desc
        key = (b,) + tuple(x.data_ptr() for x in xs)
        hit = self._descs.get(key)
        if hit is None:
            for x in xs:
                if x.stride(-1) != 1 or x.data_ptr() % 8:
                    raise ValueError("grouped gather needs contiguous, 8-byte aligned activations")
            n = len(self.layers)
            d = (_lib.QuadLinearDesc * n)(*[linear_desc(x.view(1, -1), l, None) for x, l in zip(xs, self.layers)])
            rows = (ctypes.c_int64 * n)(*[c + r0 for c, r0 in zip(self.cols, self.row0s)])
            _, outs, flags = self._args[b]
            hit = self._descs[key] = (d, rows, outs, flags, list(xs))
        return hit

    def __call__(self, xs, b: int, stream=None) -> torch.Tensor:
        from . import _lib
        s = stream if stream is not None else torch.cuda.current_stream(self.peers.device).cuda_stream
        if self.single_launch:
            d, rows, outs, flags, _ = self._group_args(xs, b)
            rc = self._lib.pp_quad_linear_group_gather(len(self.layers), d, self.peers.world, outs, self.total, rows,
                                                       flags, self.peers.epoch_ptr(b), self.ws.data_ptr(),
                                                       self.ws.numel(), s)
            if rc:
                _lib.check(rc)
            self.peers.wait(b, s)
            return self.peers.view(b)[:4 * self.total].view(4, self.total)
        for x, a in zip(xs, self._args[b][0]):
            rc = self._lib.pp_quad_linear_gather(x.data_ptr(), x.stride(-1), *a, self.ws.data_ptr(),
                                                 self.ws.numel(), s)
            if rc:
                _lib.check(rc)
        self.peers.wait(b, s)
        return self.peers.view(b)[:4 * self.total].view(4, self.total)


# ---------------------------------------------------------- graphed step ----
class GraphedStep:
    """One serving step from pinned host memory to pinned host memory,
    replayed from a single CUDA graph.

    The graph holds the copy of ``host_in`` into ``dev_in``, ``fn()`` (which
    reads ``dev_in`` and returns the device tensor of the step's result) and
    the copy of that result into a pinned host buffer, so a call costs one
    graph launch instead of one library call per Linear.  ``fn`` must be
    capturable: fixed buffers and no host synchronisation, as the groups of
    this module and ``quad_linear`` with a preallocated ``out`` are.  It runs
    once on ``stream`` before the capture (argument caches, workspaces).
    A call returns the pinned host result; read it after synchronising the
    stream the call ran on (the current stream).
    """

    def __init__(self, fn: Callable[[], torch.Tensor], host_in: torch.Tensor, dev_in: torch.Tensor,
                 stream: torch.cuda.Stream):
        if not host_in.is_pinned():
            raise ValueError("host_in must be pinned")
        if host_in.shape != dev_in.shape or host_in.dtype != dev_in.dtype:
            raise ValueError("host_in and dev_in must match in shape and dtype")
        self.host_in, self.dev_in = host_in, dev_in
        with torch.cuda.stream(stream):
            dev_in.copy_(host_in, non_blocking=True)
            y = fn()
        stream.synchronize()
        self.host_out = torch.empty(y.shape, dtype=y.dtype).pin_memory()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=stream):
            dev_in.copy_(host_in, non_blocking=True)
            y = fn()
            self.host_out.copy_(y, non_blocking=True)

    def __call__(self) -> torch.Tensor:
        self.graph.replay()
        return self.host_out

