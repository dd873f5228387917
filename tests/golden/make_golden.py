#!/usr/bin/env python3
"""Generate the golden fixtures in this folder by running the REFERENCE itself.

Run in a container that has the reference checkout (pure Python) available:

    python tests/golden/make_golden.py --reference <path to polar_pack checkout>

Nothing at test time reads the reference; the tests read only the ``.npz``
files written here.  What each fixture holds:

quad_layer.npz   reference ``pack_quad_layer`` (quad_kernels.py:16-50) on
                 seeded correlated weights, and the reference Triton kernel
                 ``quad_bitpacked_kernel`` (quad_kernels.py:68-143) run under
                 the Triton CPU interpreter: outputs for random activations,
                 and the decoded FP16 weights (activations = identity,
                 scales = 1).
dual_layer.npz   the same for ``quantize_polar_bitpacked`` /
                 ``polar_dual_bitpacked_kernel`` (polar_kernels.py:30-151).
quadpack_small.npz  a ``.quadpack`` v2 stream written by ``pack_quad``
                 (quaternion_packer.py:52-138) for four models of unequal
                 length (tails), its SHA-256, two code windows with their plug
                 entries, and ``unpack_quad`` (141-214) output on them.
dualpack_small.npz  a complete ``.dualpack`` v2 stream from
                 ``pack_dual_models_packed`` (polar_bitpack.py:93-189) with
                 unequal lengths, and ``unpack_dual_models`` (194-260) output.

Synthetic weights follow the benchmark distribution: base N(0, 0.02), per
model delta N(0, 0.002), 0.1% of entries scaled by 20, FP16 values.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def correlated_models(rng, n_models, shape, outlier_frac=0.001, outlier_scale=20.0):
    """Base N(0,0.02) + per-model delta N(0,0.002), 0.1% entries x20, as FP16."""
    base = rng.normal(0.0, 0.02, size=shape)
    out = []
    for _ in range(n_models):
        w = base + rng.normal(0.0, 0.002, size=shape)
        flat = w.reshape(-1)
        k = max(1, int(round(outlier_frac * flat.size)))
        idx = rng.choice(flat.size, size=k, replace=False)
        flat[idx] *= outlier_scale
        out.append(w.astype(np.float16))
    return out


def run_quad_kernel(qk, torch, triton, a, codes, luts, scales):
    M, K = a.shape
    N = codes.shape[1]
    outs = [torch.empty((M, N), dtype=torch.float16) for _ in range(4)]
    BM, BN, BK = 16, 32, 16
    grid = (triton.cdiv(M, BM) * triton.cdiv(N, BN),)
    qk.quad_bitpacked_kernel.fn[grid](
        a, codes, *luts, *outs, *scales, M, N, K,
        a.stride(0), a.stride(1), codes.stride(0), codes.stride(1),
        outs[0].stride(0), outs[0].stride(1), BLOCK_M=BM, BLOCK_N=BN, BLOCK_K=BK)
    return [o.numpy() for o in outs]


def run_dual_kernel(pk, torch, triton, a, packed, bmax, amp_lut, cos_lut, sin_lut):
    M, K = a.shape
    N = packed.shape[1]
    o1 = torch.empty((M, N), dtype=torch.float16)
    o2 = torch.empty_like(o1)
    BM, BN, BK = 16, 32, 16
    grid = (triton.cdiv(M, BM) * triton.cdiv(N, BN),)
    pk.polar_dual_bitpacked_kernel.fn[grid](
        a, packed, bmax, amp_lut, cos_lut, sin_lut, o1, o2, M, N, K,
        a.stride(0), a.stride(1), packed.stride(0), packed.stride(1),
        o1.stride(0), o1.stride(1), o2.stride(0), o2.stride(1), 1024, 32,
        BLOCK_M=BM, BLOCK_N=BN, BLOCK_K=BK)
    return [o1.numpy(), o2.numpy()]


def make_quad_layer(qk, torch, triton):
    rng = np.random.default_rng(0)
    data = {}
    for tag, (K, N) in {"a": (64, 96), "b": (37, 53), "c": (48, 256)}.items():
        ws = correlated_models(rng, 4, (K, N))
        codes, luts, scales = qk.pack_quad_layer(*[torch.from_numpy(w) for w in ws])
        for k in range(4):
            data[f"{tag}_w{k}"] = ws[k]
        data[f"{tag}_codes"] = codes.numpy()
        for i, t in enumerate(luts):
            data[f"{tag}_lut{i}"] = t.numpy()
        data[f"{tag}_scales"] = np.array(scales, dtype=np.float64)
        for M in (1, 5):
            a = torch.from_numpy(rng.normal(0, 1, size=(M, K)).astype(np.float16))
            outs = run_quad_kernel(qk, torch, triton, a, codes, luts, scales)
            data[f"{tag}_a{M}"] = a.numpy()
            for k in range(4):
                data[f"{tag}_out{M}_{k}"] = outs[k]
        eye = torch.eye(K, dtype=torch.float16)
        dec = run_quad_kernel(qk, torch, triton, eye, codes, luts, [1.0] * 4)
        for k in range(4):
            data[f"{tag}_dec{k}"] = dec[k]
    np.savez_compressed(HERE / "quad_layer.npz", **data)


def make_dual_layer(pk, torch, triton):
    rng = np.random.default_rng(1)
    data = {}
    for tag, (K, N) in {"a": (64, 96), "b": (37, 53)}.items():
        w1, w2 = correlated_models(rng, 2, (K, N))
        packed, bmax, amp_lut, cos_lut, sin_lut = pk.quantize_polar_bitpacked(
            torch.from_numpy(w1.astype(np.float32)), torch.from_numpy(w2.astype(np.float32)))
        data.update({f"{tag}_w0": w1, f"{tag}_w1": w2, f"{tag}_packed": packed.numpy(),
                     f"{tag}_bmax": bmax.numpy(), f"{tag}_amp_lut": amp_lut.numpy(),
                     f"{tag}_cos_lut": cos_lut.numpy(), f"{tag}_sin_lut": sin_lut.numpy()})
        for M in (1, 4):
            a = torch.from_numpy(rng.normal(0, 1, size=(M, K)).astype(np.float16))
            o = run_dual_kernel(pk, torch, triton, a, packed, bmax, amp_lut, cos_lut, sin_lut)
            data[f"{tag}_a{M}"] = a.numpy()
            data[f"{tag}_out{M}_0"], data[f"{tag}_out{M}_1"] = o
        eye = torch.eye(K, dtype=torch.float16)
        d = run_dual_kernel(pk, torch, triton, eye, packed, bmax, amp_lut, cos_lut, sin_lut)
        data[f"{tag}_dec0"], data[f"{tag}_dec1"] = d
        # pack_amp_phase on a sweep of every (amp, phase) pair
        aq = torch.arange(64).repeat_interleave(1024)
        pq = torch.arange(1024).repeat(64)
        data["amp_phase_all"] = pk.pack_amp_phase(aq, pq).numpy()
    np.savez_compressed(HERE / "dual_layer.npz", **data)


def make_quadpack(qp):
    rng = np.random.default_rng(2)
    n = 1_000_448
    extra = [0, 40, 0, 17]
    flat = correlated_models(rng, 4, (n + max(extra),))
    models = [flat[k][: n + extra[k]].astype(np.float32) for k in range(4)]
    with tempfile.TemporaryDirectory() as td:
        path = Path(td) / "small.quadpack"
        qp.pack_quad(models, path, plug_cap=0.05)
        buf = path.read_bytes()
        qp.unpack_quad(path, Path(td) / "out")
        restored = [np.fromfile(Path(td) / "out" / f"qmodel{k}_restored.dat", dtype=np.float32)
                    for k in range(4)]
    hs = qp.HEADER_SIZE
    hdr = qp.struct.unpack(qp.HEADER_FMT, buf[:hs])
    plug_n = hdr[9]
    codes = np.frombuffer(buf, np.uint32, count=n, offset=hs)
    pidx = np.frombuffer(buf, np.uint32, count=plug_n, offset=hs + 4 * n)
    pval = np.frombuffer(buf, np.float16, count=4 * plug_n, offset=hs + 4 * n + 4 * plug_n).reshape(-1, 4)
    tails_off = hs + 4 * n + 12 * plug_n
    data = {"header": np.frombuffer(buf[:hs], np.uint8), "sha256": np.array(hashlib.sha256(buf).hexdigest()),
            "size": np.array(len(buf)), "tails_raw": np.frombuffer(buf[tails_off:], np.uint8)}
    W = 4096
    for tag, (lo, hi) in {"w0": (0, W), "w1": (n - W, n)}.items():
        sel = (pidx >= lo) & (pidx < hi)
        data[f"{tag}_range"] = np.array([lo, hi])
        data[f"{tag}_codes"] = codes[lo:hi].copy()
        data[f"{tag}_pidx"] = pidx[sel].copy()
        data[f"{tag}_pval"] = pval[sel].copy()
        for k in range(4):
            data[f"{tag}_restored{k}"] = restored[k][lo:hi].copy()
    for k in range(4):
        data[f"tail_restored{k}"] = restored[k][n:].copy()
        data[f"model_len{k}"] = np.array(len(restored[k]))
    data["seed_models"] = np.array([2, n, *extra])
    np.savez_compressed(HERE / "quadpack_small.npz", **data)


def make_dualpack(bp, pp):
    rng = np.random.default_rng(3)
    n1, n2 = 10_000, 9_000
    flat = correlated_models(rng, 2, (n1,))
    w1 = flat[0].astype(np.float32)
    w2 = flat[1][:n2].astype(np.float32)
    cfg = pp.PackerConfig(chunk_size=4096)
    with tempfile.TemporaryDirectory() as td:
        f1, f2 = Path(td) / "m1.dat", Path(td) / "m2.dat"
        w1.tofile(f1)
        w2.tofile(f2)
        out = Path(td) / "small.dualpack"
        bp.pack_dual_models_packed(f1, f2, n1, n2, out, cfg)
        buf = out.read_bytes()
        r1, r2 = Path(td) / "r1.dat", Path(td) / "r2.dat"
        bp.unpack_dual_models(out, r1, r2)
        o1 = np.fromfile(r1, dtype=np.float32)
        o2 = np.fromfile(r2, dtype=np.float32)
    np.savez_compressed(HERE / "dualpack_small.npz", stream=np.frombuffer(buf, np.uint8),
                        w1=w1, w2=w2, restored1=o1, restored2=o2,
                        config=np.array([cfg.amp_bits, cfg.num_phases, cfg.mu, cfg.group_size,
                                         cfg.chunk_size]), plug_cap=np.array(cfg.plug_cap))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("POLAR_PACK_REFERENCE", ""),
                    help="path to the polar_pack reference checkout")
    args = ap.parse_args()
    if not args.reference or not Path(args.reference).is_dir():
        sys.exit("pass --reference <polar_pack checkout>")
    os.environ["TRITON_INTERPRET"] = "1"   # run the Triton kernels on the CPU
    sys.path.insert(0, str(Path(args.reference).resolve()))
    import torch
    import triton
    import quad_kernels as qk
    import polar_kernels as pk
    import quaternion_packer as qp
    import polar_bitpack as bp
    import polar_packer as pp
    torch.manual_seed(0)
    make_quad_layer(qk, torch, triton)
    make_dual_layer(pk, torch, triton)
    make_dualpack(bp, pp)
    make_quadpack(qp)
    for f in sorted(HERE.glob("*.npz")):
        print(f"{f.name}: {f.stat().st_size / 1024:.1f} KiB")


if __name__ == "__main__":
    main()
