"""Dual-pack (2-model, 16-bit polar code) oracle: numpy restatement.

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

* ``pack_amp_phase``            -- polar_kernels.py:9-11
* ``quantize_polar_bitpacked``  -- kernel-layout packer, polar_kernels.py:118-151
* ``decode_dual_fp16``          -- in-kernel decode, polar_kernels.py:64-79
* ``dual_gemm``                 -- decode + FP32-accumulate dot, no scale,
                                   polar_kernels.py:58-95
"""
from __future__ import annotations

import math

import numpy as np


def pack_amp_phase(amp_q, phase_q) -> np.ndarray:
    """``int16((amp & 63) << 10 | (phase & 1023)) - 32768``, polar_kernels.py:9-11."""
    packed = ((np.asarray(amp_q).astype(np.int32) & 0x3F) << 10) | \
        (np.asarray(phase_q).astype(np.int32) & 0x3FF)
    return (packed - 32768).astype(np.int16)


def _linspace_f32(start: float, end: float, steps: int) -> np.ndarray:
    """Float32 ``linspace`` with torch's CPU rounding.

    The first half is ``start + step*i`` and the second half
    ``end - step*(steps-1-i)``, each with one rounding (a fused multiply-add);
    ``step`` is the float32 quotient.  This reproduces
    ``torch.linspace(-pi, pi, P+1)`` bit for bit (polar_kernels.py:145),
    which numpy's float64 ``linspace`` does not.
    """
    s32, e32 = np.float32(start), np.float32(end)
    step = np.float64((e32 - s32) / np.float32(steps - 1))
    idx = np.arange(steps, dtype=np.float64)
    lo = (np.float64(s32) + step * idx).astype(np.float32)
    hi = (np.float64(e32) - step * (steps - 1 - idx)).astype(np.float32)
    return np.where(np.arange(steps) < steps // 2, lo, hi)


def dual_luts(amp_bits: int = 6, num_phases: int = 1024, mu: float = 255):
    """``amp_lut[2^amp_bits]``, ``cos_lut``, ``sin_lut`` FP16, polar_kernels.py:145-149."""
    levels = (1 << amp_bits) - 1
    log_mu = math.log(1 + mu)
    phases = _linspace_f32(-math.pi, math.pi, num_phases + 1)[:-1]
    cos_lut = np.cos(phases).astype(np.float16)
    sin_lut = np.sin(phases).astype(np.float16)
    i = np.arange(levels + 1, dtype=np.float32)
    amp_lut = ((np.exp(i / np.float32(levels) * np.float32(log_mu)) - np.float32(1.0))
               / np.float32(mu)).astype(np.float16)
    return amp_lut, cos_lut, sin_lut


def quantize_polar_bitpacked(w1, w2, amp_bits=6, num_phases=1024, mu=255, group_size=32):
    """Restates polar_kernels.py:118-151 in float32 numpy.

    Returns ``(packed int16 (K,N), bmax fp16[G], amp_lut, cos_lut, sin_lut)``.
    """
    w1 = np.asarray(w1, dtype=np.float32)
    w2 = np.asarray(w2, dtype=np.float32)
    K, N = w1.shape
    amplitude = np.sqrt(w1 ** 2 + w2 ** 2)
    phase = np.arctan2(w2, w1)
    phase_q = (np.round((phase + np.float32(math.pi)) / np.float32(2 * math.pi) * num_phases)
               .astype(np.int64) % num_phases).astype(np.int16)
    total = K * N
    amp_flat = amplitude.ravel()
    pad = (group_size - total % group_size) % group_size
    if pad:
        amp_flat = np.pad(amp_flat, (0, pad))
    grouped = amp_flat.reshape(-1, group_size)
    bmax = np.abs(grouped).max(axis=1, keepdims=True)
    bmax = np.where(bmax > 1e-10, bmax, np.float32(1.0)).astype(np.float32)
    norm = grouped / bmax
    log_mu = np.float32(math.log(1 + mu))
    compressed = np.sign(norm) * np.log1p(np.float32(mu) * np.abs(norm)) / log_mu
    levels = (1 << amp_bits) - 1
    amp_q = np.clip(np.round(compressed * levels), 0, levels).astype(np.int8).ravel()[:total].reshape(K, N)
    packed = pack_amp_phase(amp_q, phase_q)
    amp_lut, cos_lut, sin_lut = dual_luts(amp_bits, num_phases, mu)
    return packed, bmax.ravel().astype(np.float16), amp_lut, cos_lut, sin_lut


def decode_dual_fp16(packed, bmax, amp_lut, cos_lut, sin_lut, group_size=32,
                     group_index=None, amp_override=None):
    """Decode int16 codes ``(K,N)`` into two FP16 arrays.

    Restates polar_kernels.py:64-79: ``u = p + 32768``, ``amp = (u>>10)&63``,
    ``ph = u & 1023``; ``amplitude = fp32(amp_lut[amp]) * fp32(bmax[g])`` with
    ``g = (k*N + n) // group_size`` (flat row-major index); then
    ``b1 = fp16(amplitude * fp32(cos_lut[ph]))`` and the same with ``sin``.

    ``group_index`` overrides ``g`` (file streams index groups by their flat
    stream position); ``amp_override`` is an ``(mask, fp32 values)`` pair that
    replaces the amplitude where a plug applies (polar_bitpack.py:240-242).
    """
    p = np.asarray(packed).astype(np.int32)
    K, N = p.shape
    u = p + 32768
    amp_q = (u >> 10) & 0x3F
    ph = u & 0x3FF
    if group_index is None:
        group_index = (np.arange(K, dtype=np.int64)[:, None] * N
                       + np.arange(N, dtype=np.int64)[None, :]) // group_size
    amp = np.asarray(amp_lut, np.float16)[amp_q].astype(np.float32) * \
        np.asarray(bmax, np.float16)[group_index].astype(np.float32)
    if amp_override is not None:
        mask, vals = amp_override
        amp = np.where(mask, np.asarray(vals, np.float32), amp)
    cos_v = np.asarray(cos_lut, np.float16)[ph].astype(np.float32)
    sin_v = np.asarray(sin_lut, np.float16)[ph].astype(np.float32)
    return [(amp * cos_v).astype(np.float16), (amp * sin_v).astype(np.float16)]


def dual_gemm(a, packed, bmax, amp_lut, cos_lut, sin_lut, group_size=32, decoded=None):
    """``out_j = fp16(a @ B_j)`` with float64 accumulation, polar_kernels.py:81-95."""
    bs = decoded if decoded is not None else decode_dual_fp16(
        packed, bmax, amp_lut, cos_lut, sin_lut, group_size)
    a64 = np.asarray(a, dtype=np.float16).astype(np.float64)
    return [(a64 @ b.astype(np.float64)).astype(np.float32).astype(np.float16) for b in bs]
