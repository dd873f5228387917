#!/usr/bin/env python3
"""Benchmark of the fused quad dequant-GEMV on 1..8 B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: the quad-pack single-layer sweep -- four correlated synthetic models
(base N(0,0.02) + delta N(0,0.002), 0.1% entries x20, FP16), packed into
``.quadpack`` v2 streams (plug cap 5%), Linear shapes in x out = 2048x2048,
2048x11008, 11008x2048, 2048x256, batch 1.  One step = the four Linears
(4 outputs per pass over the codes), run as ONE grouped launch
(``QuadLinearGroup``: each Linear on its share of the SMs, plug correction
fused).  R = 4 replica streams rotate step to step, so each step reads
~230 MB of codes last touched ~690 MB earlier: inputs exceed the 126 MB L2
and no flush is needed.  Kernels run with launch overlap (programmatic
dependent launch) unless ``--no-overlap``.

Further legs (in ``config``): real 4-model decode steps of the 3B-class
(configs[2]) and 7B-class decoders at batch 1 per model
(``decode_step_3b`` / ``decode_step_7b``; ``--no-decode``, ``--no-7b``), the
dual-pack kernel on the sweep shapes (``dual_gemv_b1``; ``--no-dual``) and the
quad path at 16 and 64 batch rows (configs[3]; ``batched_rows``;
``--no-batched``).

Metric: packed-stream GB/s = algorithmic bytes / device time, where the
bytes of one Linear are 4*N*K (codes) + 12*P (plug index + values) +
2*M*K (activations) + 8*M*N (four FP16 outputs).  The roofline entry is the
step's grouped launch (the only kernel of the step).

With N > 1 GPUs (launched by torch.distributed.run) each Linear is
row-sharded (column-parallel): rank r owns output rows [r*N/P, (r+1)*N/P),
a contiguous slice of the file-layout stream.  The GEMVs store their rows
straight into every rank's buffer over NVLink (peer memory), the sweep's
four Linears as one grouped launch that publishes once, then one bounded
wait per step (``--nccl-gather``: one NCCL all-gather per step instead).
Each rank's gathered outputs are checked against the unsharded Linears
before timing.  Total work is fixed (strong scaling); time is the max over
ranks of CUDA-event time.

``--impl reference`` times the reference's own CPU path (the oracle's
restatement of ``unpack_quad`` -- float64 decode, plug merge, scale -- then a
host matmul) on a bounded row sample of the same shapes, all host threads.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

SHAPES = [(2048, 2048), (2048, 11008), (11008, 2048), (2048, 256)]  # (in K, out N)
METRIC = "fused quad dequant-GEMV GB/s (% HBM peak); 4-model decode tok/s @1-8 GPU"
UNIT = "GB/s"
WORKLOAD = "quad-pack single-layer sweep (BASELINE configs[1]): Linear in x out 2048x2048, 2048x11008, " \
           "11008x2048, 2048x256, batch 1, 4 correlated models, .quadpack plug cap 5%"
HBM_FALLBACK = 6650.0


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return HBM_FALLBACK, "fallback"


def layer_bytes(N, K, P, M):
    return 4 * N * K + 12 * P + 2 * M * K + 8 * M * N


# ------------------------------------------------------------ clocks ----
class ClockSampler:
    """nvidia-smi samples during the timed region (SM clock, throttle reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# 3B-class dense decoder of BASELINE configs[2] (hidden 2048, intermediate
# 11008, 16 q / 2 kv heads of 128, vocab 151936, 36 layers)
DECODE_3B = {"layers": 36, "hidden": 2048, "inter": 11008, "q_heads": 16, "kv_heads": 2, "head_dim": 128,
             "vocab": 151936}


# 7B-class dense decoder of BASELINE configs[4] (hidden 3584, intermediate
# 18944, 28 q / 4 kv heads of 128, vocab 152064, 28 layers)
DECODE_7B = {"layers": 28, "hidden": 3584, "inter": 18944, "q_heads": 28, "kv_heads": 4, "head_dim": 128,
             "vocab": 152064}


# ------------------------------------------------------------ workload ----
def synth_models(torch, n, seed, device):
    """Four correlated FP16 models of length n (BASELINE distribution)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    base = torch.randn(n, generator=g, device=device, dtype=torch.float32) * 0.02
    out = []
    for _ in range(4):
        w = base + torch.randn(n, generator=g, device=device, dtype=torch.float32) * 0.002
        k = max(1, n // 1000)
        idx = torch.randint(0, n, (k,), generator=g, device=device)
        w[idx] *= 20
        out.append(w.half())
    del base
    return out


def build_streams(torch, replicas, device, shapes=SHAPES):
    from polar_pack_b200.quadpack import DevicePackedStream, pack_quad_device
    n = sum(N * K for K, N in shapes)
    streams = []
    for r in range(replicas):
        models = synth_models(torch, n, 1000 + r, device)
        p = pack_quad_device(models, plug_cap=0.05, seed=42, windows=16, window=1_000_000)
        del models
        streams.append(DevicePackedStream(p))
        torch.cuda.empty_cache()
    return streams


def layer_slices(stream, shapes, rank, world):
    """Row shard [rank*N/world, (rank+1)*N/world) of every Linear of a stream."""
    res, off = [], 0
    for K, N in shapes:
        n0, n1 = N * rank // world, N * (rank + 1) // world
        res.append(stream.linear(off + n0 * K, n1 - n0, K))
        off += N * K
    return res


# ------------------------------------------------------------ our arm ----
def run_ours(args):
    import torch
    import torch.distributed as dist
    from polar_pack_b200 import _lib
    from polar_pack_b200.quadpack import quad_linear, quad_linear_workspace_bytes

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    M = args.batch
    _lib.set_launch_overlap(not args.no_overlap)
    if args.decode_only:
        run_decode_only(torch, dist, dev, args, world, rank)
        return
    streams = build_streams(torch, args.replicas, dev)
    sets = [layer_slices(s, SHAPES, rank, world) for s in streams]
    for s in streams:
        s.check_plug_index()
    full_sets = [layer_slices(s, SHAPES, 0, 1) for s in streams] if world > 1 else sets

    lib = _lib.load()
    # everything runs on one side stream, which is also the graph-capture stream
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    sh = stream.cuda_stream
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    xs = [torch.randn(M, K, generator=g, device=dev).half() for K, _ in SHAPES]
    ws_bytes = max(quad_linear_workspace_bytes(M, l.N, l.K) for st in sets for l in st)
    ws = torch.zeros(max(ws_bytes, 256), dtype=torch.uint8, device=dev)

    # pre-built C-ABI argument tuples: no Python allocation inside the timed loop.
    # With N > 1 GPUs the four Linears of a step are independent, so their
    # outputs go straight into one send buffer (column block per Linear,
    # strided outputs) and ONE all-gather per step collects every rank's rows.
    calls, gathers = [], []
    for st in sets:
        row = []
        widths = [l.N for l in st]
        send = torch.zeros((4, M, sum(widths)), dtype=torch.float16, device=dev)
        col = 0
        for l, x in zip(st, xs):
            outs = [send[k, :, col:col + l.N] for k in range(4)]
            col += l.N
            pk = l.pack
            args_c = (x.data_ptr(), x.stride(0), x.stride(1), l.codes.data_ptr(), l.K,
                      _lib.ptr(l.plug_idx), _lib.ptr(l.plug_vals), _lib.ptr(l.plug_window_base),
                      ctypes.c_uint32(l.offset & 0xFFFFFFFF),
                      _lib.ptr(l.unit_plugs), _lib.ptr(l.unit_plug_off),
                      pk.tables.data_ptr(), _lib.floats4(pk.scales), _lib.ptrs(outs, 4),
                      outs[0].stride(0), outs[0].stride(1), M, l.N, l.K, ws.data_ptr(), ws.numel(), sh)
            row.append((args_c, outs, l))
        calls.append(row)
        recv = torch.empty((world * 4, M, sum(widths)), dtype=torch.float16, device=dev) if world > 1 else None
        gathers.append((send, recv))

    def launch(args_c):
        rc = lib.pp_quad_linear_fused(*args_c)
        if rc:
            _lib.check(rc)

    # the step's independent Linears as one grouped launch per replica set
    # (pp_quad_linear_group: each Linear on its share of the SMs)
    from polar_pack_b200.quadpack import QuadLinearGroup
    lgroups = [QuadLinearGroup([l for _, _, l in row], xs, [outs for _, outs, _ in row]) for row in calls]

    # N > 1 GPUs at batch 1: every rank's GEMVs store their rows straight into
    # all ranks' gather buffers (peer memory over NVLink) and one bounded wait
    # per step makes the stream wait for every rank; two buffers alternate
    use_peer = world > 1 and M == 1 and not args.nccl_gather
    peers, pgroups = None, []
    if use_peer:
        from polar_pack_b200.parallel import PeerBuffers, PeerShardedGroup, row_shard
        Ns = [N for _, N in SHAPES]
        peers = PeerBuffers(4 * sum(Ns), nbuf=2, device=dev)
        r0s = [row_shard(N, world, rank)[0] for N in Ns]
        pgroups = [PeerShardedGroup(st, Ns, r0s, peers) for st in sets]

    def step(i):
        if use_peer:
            pgroups[i % len(pgroups)](xs, i % 2, sh)
            return
        lgroups[i % len(lgroups)](sh)
        if world > 1:
            send, recv = gathers[i % len(gathers)]
            dist.all_gather_into_tensor(recv, send)   # the 4 models' row shards of all 4 Linears

    per_step_bytes = sum(layer_bytes(l.N, l.K, l.p_hi - l.p_lo, M) for l in full_sets[0])
    avg_bytes = statistics.mean(sum(layer_bytes(l.N, l.K, l.p_hi - l.p_lo, M) for l in fs) for fs in full_sets)

    # correctness gate before timing: the pre-built launch vs the public API
    # path (same kernel and partition: bit-identical), then the grouped
    # launch of the step vs the separate launches (each member has its own
    # CTA share, so its split-K order differs: within the tests' tolerance)
    ref = quad_linear(xs[0], sets[0][0])
    launch(calls[0][0][0])
    torch.cuda.synchronize(dev)
    for k in range(4):
        if not torch.equal(ref[k], calls[0][0][1][k]):
            raise RuntimeError("pre-built launch disagrees with the public API")
    lgroups[0](sh)
    torch.cuda.synchronize(dev)
    for j, (args_c, outs, l) in enumerate(calls[0]):
        ref = quad_linear(xs[j], l)
        for k in range(4):
            den = float(ref[k].double().abs().max()) or 1.0
            if float((outs[k].double() - ref[k].double()).abs().max()) / den > 1e-3:
                raise RuntimeError("grouped launch disagrees with the separate launches")

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)
    parity = gathered_parity(torch, dist, step, sets, full_sets, xs, pgroups, gathers, world, dev, M) \
        if world > 1 else None

    # one CUDA graph per replica set: the timed loop replays whole steps, so
    # host launch latency is not part of the measurement
    graphs = []
    use_graphs = not args.eager
    if use_graphs:
        try:
            for r in range(len(calls)):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    step(r)
                graphs.append(g)
            for g in graphs:
                g.replay()
            torch.cuda.synchronize(dev)
        except Exception as e:  # capture unsupported (e.g. collectives): time eager launches
            print(f"graph capture failed, timing eager launches: {e}", file=sys.stderr)
            graphs, use_graphs = [], False
    if world > 1:
        dist.barrier()

    K_steps = args.steps
    # one grouped launch per step when the group runs as one (batch 1, unit
    # plugs); else one fused launch per Linear, plus a plug-correction launch
    # above batch 1
    one = (pgroups[0].single_launch if use_peer else lgroups[0].single_launch)
    launches_per_step = (1 if one else sum(1 if (l.unit_plugs is not None and M == 1) or l.plug_vals is None
                                           else 2 for l in sets[0])) + (1 if use_peer else 0)   # + the gather wait
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    t0.record(stream)
    for i in range(K_steps):
        if use_graphs:
            graphs[(args.warmup + i) % len(graphs)].replay()
        else:
            step(args.warmup + i)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        if peers is not None:   # a bounded gather wait that gave up during the timed steps fails the run
            st_ = torch.tensor([int(peers.status.item())], dtype=torch.int64, device=dev)
            dist.all_reduce(st_, op=dist.ReduceOp.MAX)
            parity["wait_status_after_timing"] = int(st_.item())
            if int(st_.item()) != 0:
                raise RuntimeError(f"a gather wait gave up during the timed steps (status {int(st_.item())})")
    total_bytes = avg_bytes * K_steps
    value = total_bytes / (ms * 1e-3) / 1e9

    # the dominant kernel alone, per shape: a graph of its launches over the
    # replica streams (rotating, so every launch reads codes L2 does not hold)
    per_shape, kernel_bytes, kernel_ms = {}, 0.0, 0.0
    for j, (K, N) in enumerate(SHAPES):
        gemv_args = []
        for st in sets:
            l = st[j]
            outs = [torch.empty((M, l.N), dtype=torch.float16, device=dev) for _ in range(4)]
            gemv_args.append((xs[j].data_ptr(), xs[j].stride(0), xs[j].stride(1), l.codes.data_ptr(), l.K,
                              _lib.ptr(l.plug_idx), _lib.ptr(l.plug_vals), _lib.ptr(l.plug_window_base),
                              ctypes.c_uint32(l.offset & 0xFFFFFFFF), _lib.ptr(l.unit_plugs),
                              _lib.ptr(l.unit_plug_off), l.pack.tables.data_ptr(), _lib.floats4(l.pack.scales),
                              _lib.ptrs(outs, 4), outs[0].stride(0), outs[0].stride(1), M, l.N, l.K,
                              ws.data_ptr(), ws.numel(), sh, outs))
        def gemv_pass():
            for a_ in gemv_args:
                _lib.check(lib.pp_quad_linear_fused(*a_[:-1]))
        gemv_pass()
        reps = max(4, K_steps // 2)
        torch.cuda.synchronize(dev)
        if use_graphs:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                gemv_pass()
            g.replay()
            torch.cuda.synchronize(dev)
            run = g.replay
        else:
            run = gemv_pass
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            run()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        tj = e0.elapsed_time(e1) / (reps * len(sets))
        bj = statistics.mean(layer_bytes(st[j].N, st[j].K, st[j].p_hi - st[j].p_lo, M) for st in sets)
        per_shape[f"{K}x{N}"] = {"us": round(tj * 1e3, 2), "GB/s": round(bj / (tj * 1e-3) / 1e9, 1)}
        kernel_bytes += bj
        kernel_ms += tj

    # e2e through the public API with host buffers (pinned), 1 GPU view of rank's work
    e2e = run_e2e(torch, dist, sets, xs, dev, args, world, M, full_sets, pgroups)

    # the second half of the metric: 4-model decode tokens/s of a 3B-class step
    decode = decode7 = None
    if not args.no_decode and not args.shapes and M == 1:
        decode = run_real_decode(torch, dist, dev, args, stream, DECODE_3B, ctx=1024, seed=3000, world=world,
                                 rank=rank)
        if not args.no_7b:
            decode7 = run_real_decode(torch, dist, dev, args, stream, DECODE_7B, ctx=1024, seed=7000, world=world,
                                      rank=rank)
    # batched rows on the same shapes (one GPU's kernel time)
    batched = None
    if not args.no_batched and M == 1:
        batched = run_batched_leg(torch, dev, args, lib, stream, sets)
    # the dual-pack kernel on the same shapes (one GPU's kernel time)
    dual = None
    if not args.no_dual and M == 1:
        dual = run_dual_leg(torch, dev, args, lib, stream)

    peak, peak_kind = measured_peak()
    if one and world == 1:
        # the step is one grouped launch: the dominant (only) kernel is timed
        # by the step loop itself (back-to-back launches, CUDA events)
        achieved = avg_bytes / (ms / K_steps * 1e-3) / 1e9
        roof_kernel = "quad_group_kernel<NK=1,NB=1,PLUG=1> (the step's 4 Linears in one launch, plugs fused)"
        roof_from = ("algorithmic bytes (4NK + 12P + 2MK + 8MN) of the 4 Linears / the per-launch CUDA-event time "
                     "of the timed steps (one launch per step)")
    else:
        achieved = kernel_bytes / (kernel_ms * 1e-3) / 1e9
        roof_kernel = "quad_gemv_kernel<NK=1,NB=1,PLUG=1> (file layout, batch 1, plugs fused)"
        roof_from = ("algorithmic bytes (4NK + 12P + 2MK + 8MN) over the 4 shapes / their per-launch CUDA-event "
                     "time (graph of back-to-back launches)")
    traffic = load_traffic() if (one and world == 1) else load_traffic("dram_bytes_per_launch_2048x11008_fused")
    res = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": K_steps,
        "warmup": args.warmup, "ms_per_step": round(ms / K_steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "u32 codes -> fp16 weights, fp32 accumulate",
        "data": "synthetic (seeded random-init correlated weights; no checkpoints available)",
        "config": {"workload": WORKLOAD if not args.shapes else f"subset {args.shapes} of: {WORKLOAD}",
                   "batch": M, "replica_streams": args.replicas,
                   "bytes_per_step": int(per_step_bytes), "l2": "inputs per step ~200 MB > 126 MB L2, "
                   "4 rotating replica streams (no flush)",
                   "parallelism": (f"row-sharded x{world}, outputs stored into every rank's buffer over NVLink "
                                   "by the GEMV, one gather wait per step" if use_peer else
                                   f"row-sharded x{world}, one NCCL all-gather per step") if world > 1
                                  else "single GPU",
                   "timing": ("CUDA graph replay of whole steps" if use_graphs else "eager launches") +
                             ("; launch overlap on" if not args.no_overlap else ""),
                   "per_shape_gemv_kernel": per_shape,
                   "parity": parity,
                   "decode_step_3b": decode,
                   "decode_step_7b": decode7,
                   "dual_gemv_b1": dual,
                   "batched_rows": batched},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} hbm_gbs",
                     "kernel": roof_kernel, "achieved_from": roof_from,
                     "traffic": traffic,
                     "traffic_of": ("one grouped launch of the step (ncu dram read + write; algorithmic "
                                    f"{avg_bytes / 1e6:.1f} MB)") if (one and world == 1) else
                                   "one 2048x11008 launch (ncu dram read + write)"},
        "e2e": e2e,
        "gpu_launches": launches_per_step * K_steps,
        "gpu_launches_note": ("per step: one grouped launch of the 4 Linears (plug correction fused)" if one else
                              "per Linear: the GEMV kernel with the plug correction fused in (batch 1)") +
                             ("; per step: one gather wait kernel" if use_peer else ""),
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline(streams[0], M, budget_s=args.cpu_seconds)
    # graphs that hold NCCL calls must be released before the process group
    graphs.clear()
    torch.cuda.synchronize(dev)
    if peers is not None:
        peers.close()   # unmaps the peers' buffers once no rank writes into them
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res))


def gathered_parity(torch, dist, step, sets, full_sets, xs, pgroups, gathers, world, dev, M):
    """One gathered step on every rank against the full (unsharded) Linears
    on this GPU; raises on a mismatch so that a multi-GPU line always
    carries a checked result.  The shards' split-K order differs from the
    full Linear's, so the bar is the tests' tolerance, not bit equality."""
    from polar_pack_b200.parallel import row_shard
    from polar_pack_b200.quadpack import quad_linear
    step(0)
    torch.cuda.synchronize(dev)
    if pgroups:
        res = pgroups[0].peers.view(0)[:4 * pgroups[0].total].view(4, 1, -1).clone()
        cols = pgroups[0].cols
        got = [[res[k, :, cols[j]:cols[j] + l.N] for k in range(4)] for j, l in enumerate(full_sets[0])]
        status = int(pgroups[0].peers.status.item())
    else:
        send, recv = gathers[0]
        rv = recv.view(world, 4, M, -1)
        got, col = [], 0
        for l in full_sets[0]:
            w = -(-l.N // world)
            got.append([torch.cat([rv[r, k, :, col:col + row_shard(l.N, world, r)[1] - row_shard(l.N, world, r)[0]]
                                   for r in range(world)], dim=1) for k in range(4)])
            col += w
        status = 0
    worst = 0.0
    for j, l in enumerate(full_sets[0]):
        ref = quad_linear(xs[j], l)
        for k in range(4):
            den = float(ref[k].double().abs().max())
            err = float((got[j][k].double() - ref[k].double()).abs().max()) / (den if den > 0 else 1.0)
            worst = max(worst, err)
    t = torch.tensor([worst, float(status)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    worst, status = float(t[0]), int(t[1])
    ok = worst <= 1e-3 and status == 0
    if not ok:
        raise RuntimeError(f"gathered outputs disagree with the full Linears: max rel err {worst:.3g}, "
                           f"wait status {status}")
    return {"ok": True, "max_rel_err": worst, "wait_status": status, "ranks_checked": world,
            "what": "every rank's gathered outputs of one step vs the unsharded Linears on its GPU "
                    "(max over ranks and models of max|y-y_full|/max|y_full|, bar 1e-3)"}


def run_batched_leg(torch, dev, args, lib, stream, sets, rows=(16, 64)):
    """configs[3]-style batched rows on the sweep shapes, through the same
    entry point as the step (pp_quad_linear_fused; above one row the plug
    correction is its own kernel).  At more than 16 rows and N or K >= 4096
    the tcgen05 tile kernel runs, else the mma.sync GEMV in 16-row chunks.
    Per shape: a graph of back-to-back calls over the replica streams."""
    from polar_pack_b200 import _lib
    from polar_pack_b200.quadpack import quad_linear_workspace_bytes
    sh = stream.cuda_stream
    g = torch.Generator(device=dev)
    g.manual_seed(31)
    res = {}
    for M in rows:
        per_shape, tot_b, tot_f, tot_t = {}, 0.0, 0.0, 0.0
        for j, (K, N) in enumerate(SHAPES):
            x = torch.randn(M, K, generator=g, device=dev).half()
            nb = max(quad_linear_workspace_bytes(M, st[j].N, st[j].K) for st in sets)
            ws = torch.zeros(max(nb, 256), dtype=torch.uint8, device=dev)
            calls, keep = [], []
            for st in sets:
                l = st[j]
                outs = [torch.empty((M, l.N), dtype=torch.float16, device=dev) for _ in range(4)]
                keep.append(outs)
                calls.append((x.data_ptr(), x.stride(0), x.stride(1), l.codes.data_ptr(), l.K,
                              _lib.ptr(l.plug_idx), _lib.ptr(l.plug_vals), _lib.ptr(l.plug_window_base),
                              ctypes.c_uint32(l.offset & 0xFFFFFFFF), _lib.ptr(l.unit_plugs),
                              _lib.ptr(l.unit_plug_off), l.pack.tables.data_ptr(), _lib.floats4(l.pack.scales),
                              _lib.ptrs(outs, 4), outs[0].stride(0), outs[0].stride(1), M, l.N, l.K,
                              ws.data_ptr(), ws.numel(), sh))

            def run():
                for c in calls:
                    rc = lib.pp_quad_linear_fused(*c)
                    if rc:
                        _lib.check(rc)
            run()
            torch.cuda.synchronize(dev)
            graph = None
            if not args.eager:
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=stream):
                    run()
                graph.replay()
                torch.cuda.synchronize(dev)
            go = graph.replay if graph is not None else run
            rounds = 6
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(rounds):
                go()
            e1.record(stream)
            torch.cuda.synchronize(dev)
            t = e0.elapsed_time(e1) / (rounds * len(calls))
            b = statistics.mean(layer_bytes(st[j].N, st[j].K, st[j].p_hi - st[j].p_lo, M) for st in sets)
            fl = 2.0 * M * K * N * 4
            path = "tcgen05" if M > 16 and (N >= 4096 or K >= 4096) else "mma.sync GEMV"
            per_shape[f"{K}x{N}"] = {"us": round(t * 1e3, 2), "GB/s": round(b / (t * 1e-3) / 1e9, 1),
                                     "TFLOP/s": round(fl / (t * 1e-3) / 1e12, 1), "path": path}
            tot_b, tot_f, tot_t = tot_b + b, tot_f + fl, tot_t + t
            del graph, calls, keep
        res[f"M{M}"] = {"per_shape": per_shape, "GB/s": round(tot_b / (tot_t * 1e-3) / 1e9, 1),
                        "TFLOP/s": round(tot_f / (tot_t * 1e-3) / 1e12, 1)}
    torch.cuda.empty_cache()
    res["what"] = ("batched rows through pp_quad_linear_fused on the sweep shapes (in x out), 4 models; "
                   "TFLOP/s = 8 M K N / time; graph of back-to-back calls over the replica streams")
    return res


def run_dual_leg(torch, dev, args, lib, stream):
    """The dual-pack kernel (polar_dual_bitpacked, 2 models of 16-bit polar
    codes, kernel layout (K, N)) on the sweep shapes at batch 1.  Each shape
    is packed once from synthetic weights of the BASELINE distribution and
    copied into enough replicas that every launch reads codes L2 does not
    hold; a graph of back-to-back launches is timed per shape.  Bytes of one
    call: 2KN (codes) + 2 ceil(KN/32) (group scales) + 2MK + 4MN."""
    from polar_pack_b200 import _lib
    from polar_pack_b200.polar_kernels import _pad_table, quantize_polar_bitpacked
    M = 1
    per_shape, tot_b, tot_t = {}, 0.0, 0.0
    g = torch.Generator(device=dev)
    g.manual_seed(21)
    sh = stream.cuda_stream
    for K, N in SHAPES:
        base = torch.randn(K, N, generator=g, device=dev) * 0.02
        w1 = base + torch.randn(K, N, generator=g, device=dev) * 0.002
        w2 = base + torch.randn(K, N, generator=g, device=dev) * 0.002
        packed, bmax, amp, cs, sn = quantize_polar_bitpacked(w1, w2)
        del base, w1, w2
        amp, cs, sn = _pad_table(amp, 64), _pad_table(cs, 1024), _pad_table(sn, 1024)
        reps = max(2, -(-(400 << 20) // (K * N * 2)))
        packs = [(packed.clone(), bmax.clone()) for _ in range(reps)]
        x = torch.randn(M, K, generator=g, device=dev).half()
        o1 = torch.empty(M, N, device=dev, dtype=torch.float16)
        o2 = torch.empty_like(o1)
        nb = _lib._size_t()
        _lib.check(lib.pp_dual_gemm_workspace_bytes(M, N, K, N, 1, ctypes.byref(nb)))
        ws = torch.zeros(max(nb.value, 256), dtype=torch.uint8, device=dev)
        calls = [(x.data_ptr(), K, 1, pk.data_ptr(), N, 1, bm.data_ptr(), 32, amp.data_ptr(), cs.data_ptr(),
                  sn.data_ptr(), o1.data_ptr(), o2.data_ptr(), N, 1, M, N, K, ws.data_ptr(), ws.numel(), sh)
                 for pk, bm in packs]

        def run():
            for c in calls:
                rc = lib.pp_dual_gemm(*c)
                if rc:
                    _lib.check(rc)
        run()
        torch.cuda.synchronize(dev)
        graph = None
        if not args.eager:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                run()
            graph.replay()
            torch.cuda.synchronize(dev)
        go = graph.replay if graph is not None else run
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        rounds = max(2, 80 // reps)
        e0.record(stream)
        for _ in range(rounds):
            go()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        t = e0.elapsed_time(e1) / (rounds * reps)
        b = 2 * K * N + 2 * (-(-K * N // 32)) + 2 * M * K + 4 * M * N
        per_shape[f"{K}x{N}"] = {"us": round(t * 1e3, 2), "GB/s": round(b / (t * 1e-3) / 1e9, 1)}
        tot_b += b
        tot_t += t
        del graph, packs, calls
        torch.cuda.empty_cache()
    peak, _ = measured_peak()
    gbs = tot_b / (tot_t * 1e-3) / 1e9
    return {"per_shape": per_shape, "GB/s": round(gbs, 1), "frac_of_measured_hbm": round(gbs / peak, 4),
            "kernel": "dual_tma_kernel (batch 1, TMA engine)", "batch": M,
            "what": "polar_dual_bitpacked on the sweep shapes (in x out), graph of back-to-back launches over "
                    "replicas larger than L2, launch overlap on"}


def run_decode_only(torch, dist, dev, args, world, rank):
    """``--decode-only``: the decode-step legs alone (for profiling them); one
    JSON line with tokens/s of the 3B-class step as ``value``."""
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    d3 = run_real_decode(torch, dist, dev, args, stream, DECODE_3B, ctx=1024, seed=3000, world=world, rank=rank)
    d7 = None if args.no_7b else run_real_decode(torch, dist, dev, args, stream, DECODE_7B, ctx=1024, seed=7000,
                                                 world=world, rank=rank)
    if rank == 0:
        print(json.dumps({"metric": "4-model decode tokens/s (3B-class step)", "value": d3["tok_s"], "unit": "tok/s",
                          "n_gpus": world, "higher_is_better": True, "data": "synthetic",
                          "config": {"decode_step_3b": d3, "decode_step_7b": d7}}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_real_decode(torch, dist, dev, args, stream, arch, ctx, seed, world=1, rank=0):
    """One real decoder step of the four packed models (BASELINE configs[2] /
    configs[4] at batch 1): every layer distinct, each model with its own
    token and hidden state, layers feeding each other, attention over a KV
    cache of about ``ctx`` positions.  The step (embedding, RMSNorm, packed
    qkv + bias, decode attention with RoPE + KV append, packed o + residual,
    RMSNorm, packed gate_up, SwiGLU, packed down + residual, final norm,
    packed lm_head) is one CUDA graph replayed per token.  With N > 1 GPUs
    every packed Linear is row-sharded and gathered by its GEMV into every
    rank's buffers over NVLink (one bounded wait per Linear); the rest runs
    on every rank.  Time: max over ranks of CUDA-event time."""
    from polar_pack_b200.decoder import DecoderConfig, DecoderExtras, QuadDecoder, qwen2_layer_map
    from polar_pack_b200.quadpack import DevicePackedStream, SyntheticModels, layer_offsets, pack_quad_generated
    cfg = DecoderConfig(layers=arch["layers"], hidden=arch["hidden"], inter=arch["inter"], q_heads=arch["q_heads"],
                        kv_heads=arch["kv_heads"], vocab=arch["vocab"], head_dim=arch["head_dim"],
                        max_pos=ctx + 64)
    lmap = qwen2_layer_map(cfg)
    n = sum(e["numel"] for e in lmap)
    t_pack = time.time()
    p = pack_quad_generated(SyntheticModels(seed, dev), n, plug_cap=0.05, seed=42, windows=16, device=dev)
    st = DevicePackedStream(p)
    del p
    torch.cuda.empty_cache()
    t_pack = time.time() - t_pack
    ex = DecoderExtras.random(cfg, dev, seed=seed + 1)
    dec = QuadDecoder(st, cfg, ex, world=world, rank=rank)
    st.check_plug_index()
    g = torch.Generator(device=dev)
    g.manual_seed(seed + 2)
    for t in dec.kc + dec.vc:   # a cache of earlier tokens: the timed steps attend about ctx positions
        t.copy_(torch.randn(t.shape, generator=g, device=dev) * 0.5)
    steps = max(3, min(args.steps, 20))
    start = ctx - steps - args.warmup - 1
    dec.pos.fill_(start)
    if world > 1:
        dist.barrier()
    dec.capture(stream)
    toks = torch.randint(0, cfg.vocab, (4,), generator=g, device=dev, dtype=torch.int32)
    for _ in range(args.warmup):
        dec.step(toks)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        dec.step(toks)
    t1.record()
    torch.cuda.synchronize(dev)
    ms = t0.elapsed_time(t1) / steps
    finite = bool(torch.isfinite(dec.logits.float()).all())
    status = int(dec.status.item()) + (int(dec.peers.status.item()) if dec.peers is not None else 0)
    if world > 1:
        t = torch.tensor([ms, 0.0 if finite else 1.0, float(status)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, finite, status = float(t[0]), float(t[1]) == 0.0, int(t[2])
    if not finite or status:
        raise RuntimeError(f"decode step produced non-finite logits or status {status}")
    # algorithmic bytes of a step: the packed Linears (codes + plug entries +
    # activations + outputs) and the KV cache read by attention
    lin_bytes = 0
    for name, off, (N, K) in layer_offsets(lmap):
        lo, hi = st._plug_range(off, off + N * K)
        lin_bytes += 4 * N * K + 12 * (hi - lo) + 2 * 4 * K + 2 * 4 * N
    kv_bytes = cfg.layers * 4 * 2 * (ctx - 1) * cfg.kv_dim * 2
    step_bytes = lin_bytes + kv_bytes
    peak, peak_kind = measured_peak()
    gbs = step_bytes / (ms * 1e-3) / 1e9
    res = {"tok_s": round(4 / (ms * 1e-3), 1), "ms_per_step": round(ms, 3), "GB/s": round(gbs, 1),
           "frac_of_measured_hbm": round(gbs / peak, 4), "bytes_per_step": int(step_bytes),
           "launches_per_step": dec.launches_per_step(), "context": ctx, "batch_per_model": 1,
           "pack_seconds": round(t_pack, 1),
           "what": f"real 4-model decode step of a {cfg.layers}-layer dense decoder (hidden {cfg.hidden}, "
                   f"intermediate {cfg.inter}, {cfg.q_heads} q / {cfg.kv_heads} kv heads, vocab {cfg.vocab}): "
                   "one token per model, each with its own hidden state; every layer distinct; embedding, RMSNorm, "
                   "packed qkv + bias, RoPE + KV append, decode attention, packed o + residual, RMSNorm, packed "
                   "gate_up, SwiGLU, packed down + residual, final norm, packed lm_head",
           "timing": "CUDA graph of one whole step, replayed per token; CUDA events"}
    if world > 1:
        res["parallelism"] = (f"row-sharded x{world}: each GEMV stores its rows into every rank's buffer over "
                              "NVLink, one bounded wait per Linear; norms and attention on every rank")
    dec.graph = None
    torch.cuda.synchronize(dev)
    dec.close()
    del dec, st, ex
    torch.cuda.empty_cache()
    return res


def run_e2e(torch, dist, sets, xs, dev, args, world, M, full_sets, pgroups=None):
    """Same metric through the public API: every step copies that step's
    inputs from pinned host memory to the GPU, runs the Linears as one
    group (RowShardedGroup on one GPU; with N > 1 GPUs each rank computes
    its row shards, gathered through peer memory by PeerShardedGroup, or by
    one NCCL all-gather with --nccl-gather), and copies the step's result
    (the four models' outputs of every Linear, gathered) back to pinned host
    memory -- one copy each way, all inside the timed region.  Except with
    --nccl-gather, a step is one GraphedStep replay (copies and launches in
    one CUDA graph)."""
    from polar_pack_b200.parallel import GraphedStep, RowShardedGroup
    from polar_pack_b200.quadpack import quad_linear
    stream = torch.cuda.current_stream(dev)
    cap = torch.cuda.Stream(dev)  # capture stream of the graphed steps
    sizes = [x.numel() for x in xs]
    hx = torch.cat([x.reshape(-1) for x in xs]).cpu().pin_memory()   # all inputs, one pinned buffer
    dxf = torch.empty_like(hx, device=dev)
    dx, o = [], 0
    for x, n in zip(xs, sizes):
        dx.append(dxf[o:o + n].view(x.shape))
        o += n
    full_n = [N for _, N in SHAPES]
    if pgroups:
        # N > 1 GPUs: the peer-gathered group; its result is complete on every
        # rank.  One graph per (group, buffer): calls alternate the buffers.
        graphs = [[GraphedStep(lambda g=g, b=b: g(dx, b), hx, dxf, cap) for b in (0, 1)] for g in pgroups]
        host_out = graphs[0][0].host_out

        def step(i):
            graphs[i % len(graphs)][i % 2]()
    elif world == 1:
        # the independent Linears as one grouped launch (QuadLinearGroup)
        # writing into one output buffer, replayed with the copies from one
        # graph per replica
        from polar_pack_b200.quadpack import QuadLinearGroup
        graphs = []
        for st in sets:
            ob = torch.empty((4, M, sum(full_n)), dtype=torch.float16, device=dev)
            outs, col = [], 0
            for l in st:
                outs.append([ob[k, :, col:col + l.N] for k in range(4)])
                col += l.N
            grp = QuadLinearGroup(st, dx, outs)
            graphs.append(GraphedStep(lambda grp=grp, ob=ob: (grp(), ob)[1], hx, dxf, cap))
        host_out = graphs[0].host_out

        def step(i):
            graphs[i % len(graphs)]()
    else:
        # the independent Linears as one row-sharded group writing into its send buffer
        groups = [RowShardedGroup([lambda x, out, l=l: quad_linear(x, l, out=out) for l in st], full_n,
                                  writes_out=True) for st in sets]
        for g_ in groups:
            g_(dx)
        host_out = torch.empty(groups[0].raw().shape, dtype=torch.float16).pin_memory()

        def step(i):
            dxf.copy_(hx, non_blocking=True)
            grp = groups[i % len(groups)]
            grp(dx)
            host_out.copy_(grp.raw(), non_blocking=True)
    h2d, d2h = hx.numel() * 2, host_out.numel() * 2

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.steps):
        step(args.warmup + i)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    ms = t0.elapsed_time(t1)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    total = 0  # whole-job bytes: the full Linears (every rank streams its row shard)
    for i in range(args.steps):
        for l in full_sets[(args.warmup + i) % len(full_sets)]:
            total += layer_bytes(l.N, l.K, l.p_hi - l.p_lo, M)
    return {"value": round(total / (ms * 1e-3) / 1e9, 1), "unit": UNIT, "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h),
            "api": "polar_pack_b200.parallel.GraphedStep of a PeerShardedGroup (grouped gathered launch)" if pgroups
                   else "polar_pack_b200.parallel.GraphedStep of a quadpack.QuadLinearGroup (one grouped launch)"
                   if world == 1 else "polar_pack_b200.parallel.RowShardedGroup of quadpack.quad_linear",
            "timing": "each step: pinned host inputs -> device, the Linears, result -> pinned host, "
                      "one CUDA graph launch per step" if (pgroups or world == 1) else "eager calls"}


def load_traffic(key="dram_bytes_per_launch_sweep_group"):
    p = ROOT / "profiles" / "quad_linear_traffic.json"
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text()).get(key)
    except Exception:
        return None


# ------------------------------------------------------ CPU reference ----
def _ref_cpu_rows(ctx, K, N, off, rows, M, x):
    """Reference CPU path on `rows` output rows of one Linear: unpack then matmul."""
    import torch
    from oracle.formats import unpack_quad_range
    codes, pos, vals, scales, r_max, pool, nthreads = ctx
    start, stop = off, off + rows * K
    bounds = np.linspace(start, stop, nthreads + 1).astype(np.int64)
    parts = list(pool.map(lambda ab: unpack_quad_range(codes, pos, vals, scales, r_max, int(ab[0]), int(ab[1])),
                          zip(bounds[:-1], bounds[1:])))
    ws = [np.concatenate([p[k] for p in parts]).reshape(rows, K) for k in range(4)]
    xt = torch.from_numpy(x.astype(np.float32))
    return [xt @ torch.from_numpy(w).T for w in ws]


def cpu_context(stream_host, nthreads):
    codes, pos, vals, scales, r_max = stream_host
    pool = cf.ThreadPoolExecutor(max_workers=nthreads)
    return (codes, pos, vals, scales, r_max, pool, nthreads)


def host_stream(stream_dev):
    return (stream_dev.codes.cpu().numpy(), stream_dev._pos_host, stream_dev.plug_vals.cpu().numpy(),
            list(stream_dev.scales), stream_dev.header.r_max)


def sample_shapes(fraction):
    """(K, rows) per sweep shape: the leading `fraction` of the output rows."""
    return [(K, max(1, int(round(N * fraction)))) for K, N in SHAPES]


def timed_ref_sample(ctx, M, layers, rng):
    """One reference step over `layers` [(K, rows, offset)]; returns (bytes, seconds)."""
    nbytes, t = 0, 0.0
    pos = ctx[1]
    for K, rows, off in layers:
        x = rng.normal(0, 1, size=(M, K)).astype(np.float16)
        s = time.perf_counter()
        _ref_cpu_rows(ctx, K, rows, off, rows, M, x)
        t += time.perf_counter() - s
        P = int(np.searchsorted(pos, off + rows * K) - np.searchsorted(pos, off))
        nbytes += layer_bytes(rows, K, P, M)
    return nbytes, t


def stream_layers(shapes_rows, full_shapes=None):
    """[(K, rows, offset)] for rows taken from the start of each Linear."""
    res, off = [], 0
    for i, (K, rows) in enumerate(shapes_rows):
        res.append((K, rows, off))
        off += (full_shapes[i][1] if full_shapes else rows) * K
    return res


def cpu_baseline(stream_dev, M, budget_s=15.0):
    import torch
    nthreads = os.cpu_count() or 1
    torch.set_num_threads(nthreads)
    ctx = cpu_context(host_stream(stream_dev), nthreads)
    rng = np.random.default_rng(0)
    fraction = 1 / 32
    layers = stream_layers(sample_shapes(fraction), SHAPES)
    total_b, total_t, steps = 0, 0.0, 0
    while total_t < budget_s and steps < 64:
        b, t = timed_ref_sample(ctx, M, layers, rng)
        total_b += b
        total_t += t
        steps += 1
    ctx[5].shutdown()
    return {"value": round(total_b / total_t / 1e9, 4), "unit": UNIT, "cores": nthreads, "kind": "port",
            "sample": f"{steps} passes over 1/32 of the output rows of each sweep shape: oracle unpack_quad "
                      f"restatement (float64 decode + plug merge + scale, {nthreads} threads) then fp32 "
                      f"torch.matmul on the host", "cpu": cpu_name()}


def cpu_name():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch
    from polar_pack_b200.quadpack import pack_quad_device
    nthreads = os.cpu_count() or 1
    torch.set_num_threads(nthreads)
    # the sampled rows of every sweep shape, synthesised and packed on the CPU
    # (same distribution and packer as our arm's streams)
    fraction = args.ref_fraction
    shapes_rows = sample_shapes(fraction)
    n = sum(K * rows for K, rows in shapes_rows)
    models = synth_models_cpu(torch, n, 1000)
    p = pack_quad_device(models, plug_cap=0.05, seed=42, windows=4, window=min(1_000_000, n // 2))
    pos = p["plug_pos"].numpy().astype(np.int64)
    stream_host = (p["codes"].numpy(), pos, p["plug_vals"].numpy(), list(p["scales"]), p["r_max"])
    ctx = cpu_context(stream_host, nthreads)
    layers = stream_layers(shapes_rows)
    rng = np.random.default_rng(0)
    for _ in range(args.warmup):
        timed_ref_sample(ctx, args.batch, layers, rng)
    tb, tt = 0, 0.0
    for _ in range(args.steps):
        b, t = timed_ref_sample(ctx, args.batch, layers, rng)
        tb += b
        tt += t
    ctx[5].shutdown()
    v = tb / tt / 1e9
    res = {"impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": UNIT, "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(tt / args.steps * 1e3, 2),
           "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
           "dtype": "float64 decode, fp32 matmul (host)", "data": "synthetic",
           "config": {"workload": WORKLOAD, "batch": args.batch, "sample": f"{fraction:.4f} of output rows"},
           "cpu_baseline": {"value": round(v, 4), "unit": UNIT, "cores": nthreads, "kind": "port",
                            "sample": f"rows [0, {fraction:.4f} N) of each sweep shape per step: oracle "
                                      "unpack_quad restatement + torch.matmul, "
                                      f"{nthreads} threads", "cpu": cpu_name()},
           "e2e": {"value": round(v, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
           "gpu_launches": 0}
    print(json.dumps(res))


def synth_models_cpu(torch, n, seed):
    g = torch.Generator()
    g.manual_seed(seed)
    base = torch.randn(n, generator=g) * 0.02
    out = []
    for _ in range(4):
        w = base + torch.randn(n, generator=g) * 0.002
        idx = torch.randint(0, n, (max(1, n // 1000),), generator=g)
        w[idx] *= 20
        out.append(w.half())
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--replicas", type=int, default=4)
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ref-fraction", type=float, default=1 / 32)
    ap.add_argument("--eager", action="store_true", help="time eager launches instead of CUDA graphs")
    ap.add_argument("--no-overlap", action="store_true", help="launch kernels without programmatic overlap")
    ap.add_argument("--no-decode", action="store_true", help="skip the decode-step legs")
    ap.add_argument("--no-7b", action="store_true", help="skip the 7B decode-step leg")
    ap.add_argument("--decode-only", action="store_true", help="run only the decode-step legs (profiling)")
    ap.add_argument("--no-dual", action="store_true", help="skip the dual-pack kernel leg")
    ap.add_argument("--no-batched", action="store_true", help="skip the batched-rows leg")
    ap.add_argument("--nccl-gather", action="store_true",
                    help="with N > 1 GPUs gather the outputs with an NCCL all-gather instead of peer stores")
    ap.add_argument("--shapes", default="", help="subset of the sweep as KxN,KxN (in x out), e.g. for profiling "
                                                 "one Linear; the line then names the subset")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.shapes:
        want = [tuple(int(v) for v in t.split("x")) for t in args.shapes.split(",")]
        bad = [w for w in want if w not in SHAPES]
        if bad:
            raise SystemExit(f"--shapes: {bad} not in the sweep {SHAPES}")
        SHAPES[:] = want
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
