""".quadpack / .dualpack codecs restated in numpy, on in-memory buffers.

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

* ``QUAD_HEADER_FMT`` / ``unpack_quad_bytes``  -- quaternion_packer.py:13-19, 141-214
* ``pack_quad_bytes``                          -- quaternion_packer.py:22-138
* ``DUAL_HEADER_FMT`` / ``unpack_dual_bytes``  -- polar_bitpack.py:26-29, 194-260
* ``pack_dual_bytes``                          -- polar_bitpack.py:34-189

The unpackers are the reference's CPU decode (float64 transcendental math,
plug merge by sorted index, per-model scale, raw FP16 tails).  They are what
``bench.py --impl reference`` times as the reference CPU path, followed by a
host matmul.
"""
from __future__ import annotations

import math
import struct

import numpy as np

# ---------------------------------------------------------------- quad ----
QUAD_MAGIC = b"QUAD"
QUAD_VERSION = 2
QUAD_MU = 255.0
QUAD_CHUNK = 100_000_000
QUAD_HEADER_FMT = "<4sBBQBBBBfQ4ff4Q"          # quaternion_packer.py:18
QUAD_HEADER_SIZE = struct.calcsize(QUAD_HEADER_FMT)   # 82 bytes


def parse_quad_header(buf) -> dict:
    """Field order of quaternion_packer.py:93-94 / 147-151."""
    h = struct.unpack(QUAD_HEADER_FMT, bytes(buf[:QUAD_HEADER_SIZE]))
    magic, ver, nm, n, nb, b1, b2, b3, mu, plug_n = h[:10]
    if magic != QUAD_MAGIC or ver != QUAD_VERSION:
        raise ValueError("not a v2 .quadpack stream")
    return dict(n_models=nm, n=n, bits=(nb, b1, b2, b3), mu=mu, plug_n=plug_n,
                scales=list(h[10:14]), r_max=h[14], tails=list(h[15:19]))


def quad_offsets(hdr: dict) -> dict:
    """Byte offsets of the sections, quaternion_packer.py:155-157."""
    codes = QUAD_HEADER_SIZE
    plug = codes + hdr["n"] * 4
    vals = plug + hdr["plug_n"] * 4
    tails = vals + hdr["plug_n"] * 8
    return dict(codes=codes, plug_idx=plug, plug_vals=vals, tails=tails)


def quad_sections(buf):
    """Zero-copy numpy views ``(hdr, codes, plug_idx, plug_vals, tails[4])``."""
    hdr = parse_quad_header(buf)
    off = quad_offsets(hdr)
    n, pn = hdr["n"], hdr["plug_n"]
    codes = np.frombuffer(buf, np.uint32, count=n, offset=off["codes"])
    pidx = np.frombuffer(buf, np.uint32, count=pn, offset=off["plug_idx"])
    pval = np.frombuffer(buf, np.float16, count=pn * 4, offset=off["plug_vals"]).reshape(-1, 4)
    tails, o = [], off["tails"]
    for t in hdr["tails"]:
        tails.append(np.frombuffer(buf, np.float16, count=t, offset=o))
        o += 2 * t
    return hdr, codes, pidx, pval, tails


def _to_hyperspherical(w1, w2, w3, w4):
    """quaternion_packer.py:22-27."""
    r = np.sqrt(w1 ** 2 + w2 ** 2 + w3 ** 2 + w4 ** 2)
    t1 = np.arctan2(np.sqrt(w2 ** 2 + w3 ** 2 + w4 ** 2), w1)
    t2 = np.arctan2(np.sqrt(w3 ** 2 + w4 ** 2), w2)
    t3 = np.mod(np.arctan2(w4, w3), 2 * np.pi)
    return r, t1, t2, t3


def quantize_quad_chunk(wc, r_max, with_err=False):
    """Codes (and the relative decode error) of one chunk, quaternion_packer.py:30-49."""
    log_mu = math.log1p(QUAD_MU)
    r, t1, t2, t3 = _to_hyperspherical(*wc)
    nq = np.round(np.log1p(QUAD_MU * r / r_max) / log_mu * 255).clip(0, 255).astype(np.uint32)
    q1 = np.round(t1 / np.pi * 255).clip(0, 255).astype(np.uint32)
    q2 = np.round(t2 / np.pi * 255).clip(0, 255).astype(np.uint32)
    q3 = np.round(t3 / (2 * np.pi) * 255).clip(0, 255).astype(np.uint32)
    codes = (nq << 24) | (q1 << 16) | (q2 << 8) | q3
    if not with_err:
        return codes
    rr = (np.exp(nq / 255 * log_mu) - 1) * r_max / QUAD_MU
    a1, a2, a3 = q1 / 255 * np.pi, q2 / 255 * np.pi, q3 / 255 * 2 * np.pi
    rw = (rr * np.cos(a1), rr * np.sin(a1) * np.cos(a2),
          rr * np.sin(a1) * np.sin(a2) * np.cos(a3), rr * np.sin(a1) * np.sin(a2) * np.sin(a3))
    err = np.sqrt(sum((wc[k] - rw[k]) ** 2 for k in range(4))) / np.maximum(r, 1e-12)
    return codes, err


def pack_quad_bytes(models, plug_cap=0.05, threshold_windows=100, window=1_000_000,
                    seed=42) -> bytes:
    """In-memory ``.quadpack`` v2 writer restating quaternion_packer.py:52-138.

    Pass A: per-model RMS on the common length; pass B: ``r_max * 1.001`` and
    the plug threshold = ``(1 - plug_cap)`` percentile of the decode error over
    ``threshold_windows`` random windows (seed 42); pass C: codes plus plugs
    (normalised FP16 4-tuples at ascending indices), then raw FP16 tails.
    ``window`` is 1M in the reference; the argument exists so that small test
    streams can be built (the reference requires ``n > 1M``).
    """
    lengths = [len(m) for m in models]
    n = min(lengths)
    tails = [int(L - n) for L in lengths]
    s = [math.sqrt(float(np.sum(np.asarray(m[:n], np.float64) ** 2)) / n) for m in models]
    wc = [np.asarray(m[:n], dtype=np.float32) / sk for m, sk in zip(models, s)]
    r_max = float(np.max(np.sqrt(sum(x ** 2 for x in wc)))) * 1.001
    rng = np.random.default_rng(seed)
    starts = rng.integers(0, n - window, threshold_windows)
    errs = [quantize_quad_chunk([x[st:st + window] for x in wc], r_max, True)[1] for st in starts]
    thr = float(np.percentile(np.concatenate(errs), (1 - plug_cap) * 100))
    codes, err = quantize_quad_chunk(wc, r_max, True)
    mask = err > thr
    pidx = np.nonzero(mask)[0].astype(np.uint32)
    pval = np.stack([wc[k][mask] for k in range(4)], axis=1).astype(np.float16)
    out = [struct.pack(QUAD_HEADER_FMT, QUAD_MAGIC, QUAD_VERSION, 4, n, 8, 8, 8, 8,
                       QUAD_MU, len(pidx), *s, r_max, *tails),
           codes.astype(np.uint32).tobytes(), pidx.tobytes(), pval.tobytes()]
    for k, m in enumerate(models):
        if tails[k]:
            out.append(np.asarray(m[n:], dtype=np.float16).tobytes())
    return b"".join(out)


def unpack_quad_bytes(buf, chunk: int = QUAD_CHUNK) -> list[np.ndarray]:
    """Reference CPU decode of a ``.quadpack`` into 4 float32 arrays.

    Restates quaternion_packer.py:141-214: float64 decode of each chunk
    (172-185), plug merge by ``searchsorted`` on the sorted plug index
    (187-193), ``* s_k`` (195-196), raw FP16 tails appended (201-210).
    """
    hdr, codes, pidx, pval, tails = quad_sections(buf)
    n, s, r_max = hdr["n"], hdr["scales"], hdr["r_max"]
    log_mu = math.log1p(QUAD_MU)
    outs = [np.empty(n + t, dtype=np.float32) for t in hdr["tails"]]
    for i in range(0, n, chunk):
        j = min(i + chunk, n)
        c = codes[i:j]
        nq, q1, q2, q3 = c >> 24, (c >> 16) & 255, (c >> 8) & 255, c & 255
        rr = (np.exp(nq / 255 * log_mu) - 1) * r_max / QUAD_MU
        t1, t2, t3 = q1 / 255 * np.pi, q2 / 255 * np.pi, q3 / 255 * 2 * np.pi
        rw = [rr * np.cos(t1), rr * np.sin(t1) * np.cos(t2),
              rr * np.sin(t1) * np.sin(t2) * np.cos(t3),
              rr * np.sin(t1) * np.sin(t2) * np.sin(t3)]
        if len(pidx):
            lo, hi = np.searchsorted(pidx, i), np.searchsorted(pidx, j)
            if hi > lo:
                pos = pidx[lo:hi].astype(np.int64) - i
                for k in range(4):
                    rw[k][pos] = pval[lo:hi, k].astype(np.float32)
        for k in range(4):
            outs[k][i:j] = rw[k] * s[k]
    for k in range(4):
        if hdr["tails"][k]:
            outs[k][n:] = tails[k].astype(np.float32)
    return outs


# ---------------------------------------------------------------- dual ----
DUAL_MAGIC = b"DUALPACK"
DUAL_VERSION = 2
DUAL_HEADER_FMT = "<8s I Q Q Q B B f I Q Q"      # polar_bitpack.py:28
DUAL_HEADER_SIZE = struct.calcsize(DUAL_HEADER_FMT)   # 62 bytes


def parse_dual_header(buf) -> dict:
    """Field order of polar_bitpack.py:29 / 197-198."""
    (magic, ver, n_pairs, n1, n2, amp_bits, phase_bits, mu, gs, chunk_size,
     plug_n) = struct.unpack(DUAL_HEADER_FMT, bytes(buf[:DUAL_HEADER_SIZE]))
    if magic != DUAL_MAGIC or ver != DUAL_VERSION:
        raise ValueError("not a v2 .dualpack stream")
    return dict(n_pairs=n_pairs, n1=n1, n2=n2, amp_bits=amp_bits, phase_bits=phase_bits,
                mu=mu, group_size=gs, chunk_size=chunk_size, plug_n=plug_n)


def dual_group_count(hdr: dict) -> int:
    """Scale count: groups restart at every chunk boundary, polar_bitpack.py:201-203."""
    ng = 0
    for s in range(0, hdr["n_pairs"], hdr["chunk_size"]):
        ng += math.ceil(min(hdr["chunk_size"], hdr["n_pairs"] - s) / hdr["group_size"])
    return ng


def dual_sections(buf):
    """``(hdr, codes_u16 (host order), scales fp16, plug_idx u32, plug_val fp16)``.

    Codes are stored big-endian per pair (polar_bitpack.py:81-88); this view
    returns them as native integers ``amp << phase_bits | phase``.
    """
    hdr = parse_dual_header(buf)
    npairs, pn = hdr["n_pairs"], hdr["plug_n"]
    ng = dual_group_count(hdr)
    o = DUAL_HEADER_SIZE
    raw = np.frombuffer(buf, np.uint8, count=2 * npairs, offset=o)
    codes = (raw[0::2].astype(np.uint32) << 8) | raw[1::2].astype(np.uint32)
    o += 2 * npairs
    scales = np.frombuffer(buf, np.float16, count=ng, offset=o)
    o += 2 * ng
    pidx = np.frombuffer(buf, np.uint32, count=pn, offset=o)
    o += 4 * pn
    pval = np.frombuffer(buf, np.float16, count=pn, offset=o)
    return hdr, codes, scales, pidx, pval


def _quantize_amplitude_codes(amp_flat, amp_bits, mu, group_size, plug_cap):
    """polar_bitpack.py:34-76 (flat codes, FP16 group max, top-error plugs)."""
    levels = 2 ** amp_bits - 1
    ol = amp_flat.size
    pad = (group_size - ol % group_size) % group_size
    if pad:
        amp_flat = np.pad(amp_flat, (0, pad))
    b = amp_flat.reshape(-1, group_size)
    bmax = np.abs(b).max(axis=1, keepdims=True)
    bmax = np.where(bmax > 1e-10, bmax, 1.0)
    log_mu = np.log1p(mu)
    compressed = np.sign(b / bmax) * np.log1p(mu * np.abs(b / bmax)) / log_mu
    amp_q2d = np.round(compressed * levels).clip(0, levels).astype(np.uint8)
    restored = np.expm1(amp_q2d.astype(np.float64) / levels * log_mu) / mu
    decoded = (restored * bmax).ravel()[:ol].copy()
    amp_q = amp_q2d.ravel()[:ol]
    pidx = np.array([], dtype=np.uint32)
    pval = np.array([], dtype=np.float16)
    if plug_cap > 0:
        core = b.ravel()[:ol]
        e = (core - decoded) ** 2
        n_plug = int(plug_cap * ol)
        if n_plug > 0:
            sel = np.argpartition(e, -n_plug)[-n_plug:]
            pidx = sel.astype(np.uint32)
            pval = core[sel].astype(np.float16)
    return amp_q, bmax.astype(np.float16).ravel(), pidx, pval


def pack_dual_bytes(w1, w2, amp_bits=6, num_phases=1024, mu=255, group_size=32,
                    chunk_size=50_000_000, plug_cap=0.03) -> bytes:
    """In-memory ``.dualpack`` v2 writer restating polar_bitpack.py:93-172."""
    n1, n2 = len(w1), len(w2)
    phase_bits = 16 - amp_bits
    max_n = max(n1, n2)
    codes_p, scales_p, pi_p, pv_p = [], [], [], []
    for start in range(0, max_n, chunk_size):
        end = min(start + chunk_size, max_n)
        a = np.asarray(w1[start:min(end, n1)], np.float32) if start < n1 else np.array([], np.float32)
        b = np.asarray(w2[start:min(end, n2)], np.float32) if start < n2 else np.array([], np.float32)
        L = max(len(a), len(b))
        a = np.pad(a, (0, L - len(a)))
        b = np.pad(b, (0, L - len(b)))
        amplitude = np.sqrt(a ** 2 + b ** 2)
        phase = np.arctan2(b, a)
        ph = (np.round((phase + np.pi) / (2 * np.pi) * num_phases).astype(np.int64)
              % num_phases).astype(np.uint32)
        amp_q, bmax16, pidx, pval = _quantize_amplitude_codes(
            amplitude, amp_bits, mu, group_size, plug_cap)
        if pidx.size:
            pi_p.append(pidx + np.uint32(start))
            pv_p.append(pval)
        comb = (amp_q.astype(np.uint32) << phase_bits) | ph
        inter = np.empty(comb.size * 2, dtype=np.uint8)
        inter[0::2] = ((comb >> 8) & 0xFF).astype(np.uint8)
        inter[1::2] = (comb & 0xFF).astype(np.uint8)
        codes_p.append(inter)
        scales_p.append(bmax16)
    pidx = np.concatenate(pi_p) if pi_p else np.array([], np.uint32)
    pval = np.concatenate(pv_p) if pv_p else np.array([], np.float16)
    order = np.argsort(pidx)
    pidx, pval = pidx[order], pval[order]
    hdr = struct.pack(DUAL_HEADER_FMT, DUAL_MAGIC, DUAL_VERSION, max_n, n1, n2, amp_bits,
                      phase_bits, float(mu), group_size, chunk_size, pidx.size)
    return b"".join([hdr, np.concatenate(codes_p).tobytes(), np.concatenate(scales_p).tobytes(),
                     pidx.tobytes(), pval.tobytes()])


def unpack_dual_bytes(buf) -> list[np.ndarray]:
    """Reference CPU decode of a ``.dualpack`` into 2 float32 arrays.

    Restates polar_bitpack.py:194-260: per chunk, ``amp = expm1(q/levels *
    ln(1+mu))/mu * scale[g]`` in float64 rounded to float32, plug amplitudes
    substituted, ``ang = ph/2^phase_bits * 2pi - pi``, ``w1 = amp cos``,
    ``w2 = amp sin``; outputs truncated to ``n1`` / ``n2``.
    """
    hdr, codes, scales, pidx, pval = dual_sections(buf)
    n_pairs, cs, gs = hdr["n_pairs"], hdr["chunk_size"], hdr["group_size"]
    levels = 2 ** hdr["amp_bits"] - 1
    log_mu = np.log1p(hdr["mu"])
    pmask = (1 << hdr["phase_bits"]) - 1
    o1 = np.empty(hdr["n1"], np.float32)
    o2 = np.empty(hdr["n2"], np.float32)
    g_off, p_lo = 0, 0
    for start in range(0, n_pairs, cs):
        end = min(start + cs, n_pairs)
        L = end - start
        c = codes[start:end]
        aq = (c >> hdr["phase_bits"]) & levels
        ph = c & pmask
        n_g = math.ceil(L / gs)
        sc = scales[g_off:g_off + n_g].astype(np.float32)
        amp = (np.expm1(aq.astype(np.float64) / levels * log_mu) / hdr["mu"]
               * np.repeat(sc, gs)[:L]).astype(np.float32)
        p_hi = int(np.searchsorted(pidx, end))
        if p_hi > p_lo:
            amp[pidx[p_lo:p_hi] - start] = pval[p_lo:p_hi].astype(np.float32)
        p_lo = p_hi
        ang = ph.astype(np.float64) / (pmask + 1) * 2 * np.pi - np.pi
        w1, w2 = amp * np.cos(ang), amp * np.sin(ang)
        if start < hdr["n1"]:
            o1[start:min(end, hdr["n1"])] = w1[:min(end, hdr["n1"]) - start]
        if start < hdr["n2"]:
            o2[start:min(end, hdr["n2"])] = w2[:min(end, hdr["n2"]) - start]
        g_off += n_g
    return [o1, o2]


def unpack_quad_range(codes, plug_pos, plug_vals, scales, r_max, start, stop) -> list[np.ndarray]:
    """The body of one ``unpack_quad`` chunk (quaternion_packer.py:172-196) on
    flat positions ``[start, stop)``: float64 decode, plug merge by
    ``searchsorted``, ``* s_k``.  Returns 4 float32 arrays.

    ``plug_pos`` are int64 positions (ascending); ``codes`` the full uint32
    code array.  Used to time the reference CPU path on a bounded sample.
    """
    log_mu = math.log1p(QUAD_MU)
    c = np.asarray(codes[start:stop])
    nq, q1, q2, q3 = c >> 24, (c >> 16) & 255, (c >> 8) & 255, c & 255
    rr = (np.exp(nq / 255 * log_mu) - 1) * r_max / QUAD_MU
    t1, t2, t3 = q1 / 255 * np.pi, q2 / 255 * np.pi, q3 / 255 * 2 * np.pi
    rw = [rr * np.cos(t1), rr * np.sin(t1) * np.cos(t2),
          rr * np.sin(t1) * np.sin(t2) * np.cos(t3),
          rr * np.sin(t1) * np.sin(t2) * np.sin(t3)]
    lo, hi = np.searchsorted(plug_pos, start), np.searchsorted(plug_pos, stop)
    if hi > lo:
        pos = plug_pos[lo:hi] - start
        for k in range(4):
            rw[k][pos] = plug_vals[lo:hi, k].astype(np.float32)
    return [(rw[k] * scales[k]).astype(np.float32) for k in range(4)]
