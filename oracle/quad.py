"""Quad-pack (4-model, uint32 code) oracle: numpy restatement of the reference.

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

The reference computes everything here with torch/Triton; this module
restates the same steps with numpy so that a test can check the CUDA path on
identical inputs:

* ``quad_luts``         -- the seven FP16 lookup tables, quad_kernels.py:39-46
* ``pack_quad_layer``   -- kernel-layout packer, quad_kernels.py:16-50
* ``decode_quad_fp16``  -- the in-kernel FP16 decode chain, quad_kernels.py:103-121
* ``quad_gemm``         -- decode + FP32-accumulate dot + per-model scale at
                           store, quad_kernels.py:97-143
"""
from __future__ import annotations

import math

import numpy as np

MU = 255.0


def quad_luts(r_max: float, mu: float = MU) -> list[np.ndarray]:
    """Seven FP16[256] tables ``(norm, cos1, sin1, cos2, sin2, cos3, sin3)``.

    Follows quad_kernels.py:39-46: float32 math on ``i = 0..255``, rounded to
    FP16 once.  ``cos1 == cos2`` and ``sin1 == sin2`` by construction.
    """
    i = np.arange(256, dtype=np.float32)
    log_mu = np.float32(math.log1p(mu))
    norm = ((np.exp(i / np.float32(255) * log_mu) - np.float32(1))
            * np.float32(r_max) / np.float32(mu)).astype(np.float16)
    ang12 = i / np.float32(255) * np.float32(math.pi)
    ang3 = i / np.float32(255) * np.float32(2 * math.pi)
    c12 = np.cos(ang12).astype(np.float16)
    s12 = np.sin(ang12).astype(np.float16)
    return [norm, c12, s12, c12.copy(), s12.copy(),
            np.cos(ang3).astype(np.float16), np.sin(ang3).astype(np.float16)]


def pack_quad_layer(w1, w2, w3, w4, mu: float = MU):
    """Kernel-layout packer, restating quad_kernels.py:16-50 in float32 numpy.

    Returns ``(codes uint32 (K,N), luts list[7] fp16[256], scales list[4])``.
    Codes can differ from the torch packer by one quantisation step where a
    float32 transcendental lands on a rounding boundary; the decode contract
    is defined given the codes, so tests compare decode bit-exactly and the
    packer only statistically.
    """
    ws = [np.asarray(w, dtype=np.float32) for w in (w1, w2, w3, w4)]
    s = [np.float32(np.sqrt(np.mean(w * w, dtype=np.float32))) for w in ws]
    wn = [w / sk for w, sk in zip(ws, s)]
    r = np.sqrt(wn[0] ** 2 + wn[1] ** 2 + wn[2] ** 2 + wn[3] ** 2)
    r_max = float(r.max()) * 1.001
    log_mu = np.float32(math.log1p(mu))
    t1 = np.arctan2(np.sqrt(wn[1] ** 2 + wn[2] ** 2 + wn[3] ** 2), wn[0])
    t2 = np.arctan2(np.sqrt(wn[2] ** 2 + wn[3] ** 2), wn[1])
    t3 = np.mod(np.arctan2(wn[3], wn[2]), np.float32(2 * math.pi))
    nq = np.clip(np.round(np.log1p(np.float32(mu) * r / np.float32(r_max)) / log_mu * 255), 0, 255)
    q1 = np.clip(np.round(t1 / np.float32(math.pi) * 255), 0, 255)
    q2 = np.clip(np.round(t2 / np.float32(math.pi) * 255), 0, 255)
    q3 = np.clip(np.round(t3 / np.float32(2 * math.pi) * 255), 0, 255)
    u = lambda x: x.astype(np.int64).astype(np.uint32)
    codes = (u(nq) << 24) | (u(q1) << 16) | (u(q2) << 8) | u(q3)
    return codes.astype(np.uint32), quad_luts(r_max, mu), [float(x) for x in s]


def decode_quad_fp16(codes: np.ndarray, luts) -> list[np.ndarray]:
    """Decode uint32 codes into four FP16 weight arrays (same shape).

    Restates quad_kernels.py:103-121 exactly: byte unpack, seven FP16 table
    reads, then the FP16 product chain ``rs = r*s1``, ``rss = rs*s2``,
    ``w1 = r*c1``, ``w2 = rs*c2``, ``w3 = rss*c3``, ``w4 = rss*s3`` with a
    round-to-nearest-even FP16 result after every product.
    """
    c = np.asarray(codes, dtype=np.uint32)
    norm, c1t, s1t, c2t, s2t, c3t, s3t = [np.asarray(t, dtype=np.float16) for t in luts]
    nq = (c >> 24) & 0xFF
    q1 = (c >> 16) & 0xFF
    q2 = (c >> 8) & 0xFF
    q3 = c & 0xFF
    r = norm[nq]
    rs = (r * s1t[q1]).astype(np.float16)
    rss = (rs * s2t[q2]).astype(np.float16)
    w1 = (r * c1t[q1]).astype(np.float16)
    w2 = (rs * c2t[q2]).astype(np.float16)
    w3 = (rss * c3t[q3]).astype(np.float16)
    w4 = (rss * s3t[q3]).astype(np.float16)
    return [w1, w2, w3, w4]


def quad_gemm(a: np.ndarray, codes: np.ndarray, luts, scales, decoded=None) -> list[np.ndarray]:
    """``out_k = fp16(fp32(a @ W_k) * s_k)`` for the four models.

    ``a`` is ``(M, K)`` FP16 and ``codes`` ``(K, N)``.  The reference
    accumulates in FP32 with ``tl.dot`` (quad_kernels.py:123-126) and scales
    in FP32 before the FP16 store (131-134); the oracle accumulates in float64
    (a tighter reference for the tolerance check), then applies the FP32
    scale and the FP16 rounding the same way.  ``decoded`` may carry weights
    that already had plug values substituted.
    """
    ws = decoded if decoded is not None else decode_quad_fp16(codes, luts)
    a64 = np.asarray(a, dtype=np.float16).astype(np.float64)
    outs = []
    for w, sk in zip(ws, scales):
        acc = (a64 @ np.asarray(w, dtype=np.float16).astype(np.float64)).astype(np.float32)
        outs.append((acc * np.float32(sk)).astype(np.float16))
    return outs


def quad_gemm_f64(a: np.ndarray, ws, scales) -> list[np.ndarray]:
    """Float64 ``s_k * (a @ W_k)`` with no output rounding (tolerance anchor)."""
    a64 = np.asarray(a, dtype=np.float16).astype(np.float64)
    return [(a64 @ np.asarray(w, dtype=np.float16).astype(np.float64)) * float(sk)
            for w, sk in zip(ws, scales)]


def rel_err(y: np.ndarray, y_ref: np.ndarray) -> float:
    """``max|y - y_ref| / max|y_ref|`` per output vector, the parity metric."""
    y = np.asarray(y, dtype=np.float64)
    y_ref = np.asarray(y_ref, dtype=np.float64)
    den = float(np.max(np.abs(y_ref))) if y_ref.size else 0.0
    num = float(np.max(np.abs(y - y_ref))) if y_ref.size else 0.0
    return num / den if den > 0 else num
