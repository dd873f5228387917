"""Dual-pack (2 models, 16-bit polar codes) -- drop-in for the reference ``polar_kernels.py``.

Same names, argument order, return types and error behaviour as
polar_kernels.py:9-151; the fused decode + 2 matmuls run in the sm_100a
kernels of ``libpolarpack_b200.so``.

int16 word: ``(amp6 << 10 | phase10) - 32768``.
"""
from __future__ import annotations

import math

import torch

from . import _lib


def pack_amp_phase(amp_q, phase_q):
    """``int16((amp & 63) << 10 | (phase & 1023)) - 32768``, polar_kernels.py:9-11."""
    packed = ((amp_q.to(torch.int32) & 0x3F) << 10) | (phase_q.to(torch.int32) & 0x3FF)
    return (packed - 32768).to(torch.int16)


def dual_luts(amp_bits=6, num_phases=1024, mu=255, device=None):
    """``(amp_lut, cos_lut, sin_lut)`` FP16, computed as polar_kernels.py:145-149."""
    levels = (1 << amp_bits) - 1
    log_mu = math.log(1 + mu)
    phases = torch.linspace(-math.pi, math.pi, num_phases + 1)[:-1]
    cos_lut = torch.cos(phases).to(torch.float16)
    sin_lut = torch.sin(phases).to(torch.float16)
    i = torch.arange(levels + 1, dtype=torch.float32)
    amp_lut = ((torch.exp(i / levels * log_mu) - 1.0) / mu).to(torch.float16)
    if device is not None:
        amp_lut, cos_lut, sin_lut = (t.to(device) for t in (amp_lut, cos_lut, sin_lut))
    return amp_lut, cos_lut, sin_lut


def quantize_polar_bitpacked(w1, w2, amp_bits=6, num_phases=1024, mu=255, group_size=32):
    """Kernel-layout packer, restating polar_kernels.py:118-151.

    Returns ``(packed int16 (K,N), bmax fp16[ceil(KN/gs)], amp_lut, cos_lut,
    sin_lut)``.  Layout producer, not on the timed path.
    """
    K, N = w1.shape
    amplitude = torch.sqrt(w1 ** 2 + w2 ** 2)
    phase = torch.atan2(w2, w1)
    phase_q = (torch.round((phase + math.pi) / (2 * math.pi) * num_phases).long()
               % num_phases).to(torch.int16)
    total = K * N
    amp_flat = amplitude.flatten()
    pad = (group_size - total % group_size) % group_size
    if pad:
        amp_flat = torch.nn.functional.pad(amp_flat, (0, pad))
    grouped = amp_flat.reshape(-1, group_size)
    bmax = grouped.abs().max(dim=1, keepdim=True).values
    bmax = torch.where(bmax > 1e-10, bmax, torch.ones_like(bmax))
    norm = grouped / bmax
    log_mu = math.log(1 + mu)
    compressed = torch.sign(norm) * torch.log1p(mu * norm.abs()) / log_mu
    levels = (1 << amp_bits) - 1
    amp_q = (torch.round(compressed * levels).clamp(0, levels)
             .to(torch.int8).flatten()[:total].reshape(K, N))
    bmax = bmax.flatten().to(torch.float16)
    packed = pack_amp_phase(amp_q, phase_q)
    amp_lut, cos_lut, sin_lut = dual_luts(amp_bits, num_phases, mu, device=w1.device)
    return packed, bmax, amp_lut, cos_lut, sin_lut


def _pad_table(t: torch.Tensor, n: int) -> torch.Tensor:
    """Kernels read the full 6-bit / 10-bit code range; shorter tables get zeros."""
    if t.dtype != torch.float16:
        raise ValueError("lookup tables must be fp16")
    t = t.contiguous()
    if t.numel() >= n:
        return t
    out = torch.zeros(n, dtype=torch.float16, device=t.device)
    out[: t.numel()] = t
    return out


def polar_dual_bitpacked(a_fp16, packed, bmax, amp_lut, cos_lut, sin_lut,
                         num_phases=1024, group_size=32):
    """``(out1, out2)`` with ``out_j = fp16(a @ B_j)`` in one pass over ``packed``.

    Drop-in for polar_kernels.py:98-115.  Like the reference kernel the phase
    mask is the fixed 10 bits (``num_phases`` is accepted and unused by the
    decode); raises ``AssertionError`` on a K mismatch.
    """
    M, K = a_fp16.shape
    K_b, N = packed.shape
    assert K == K_b
    dev = _lib.require_cuda(a_fp16, packed, bmax, amp_lut, cos_lut, sin_lut)
    if a_fp16.dtype != torch.float16 or packed.dtype != torch.int16 or bmax.dtype != torch.float16:
        raise ValueError("expected fp16 activations, int16 codes and fp16 group scales")
    if bmax.numel() < -(-K * N // group_size):
        raise ValueError("bmax has fewer entries than ceil(K*N/group_size)")
    amp_lut = _pad_table(amp_lut, 64)
    cos_lut = _pad_table(cos_lut, 1024)
    sin_lut = _pad_table(sin_lut, 1024)
    bmax = bmax.contiguous()
    out1 = torch.empty((M, N), dtype=torch.float16, device=dev)
    out2 = torch.empty_like(out1)
    lib = _lib.load()
    nbytes = _lib._size_t()
    _lib.check(lib.pp_dual_gemm_workspace_bytes(M, N, K, packed.stride(0), packed.stride(1),
                                                _lib.ctypes.byref(nbytes)))
    ws = _lib.workspace(dev, nbytes.value) if nbytes.value else None
    _lib.call("pp_dual_gemm", a_fp16.data_ptr(), a_fp16.stride(0), a_fp16.stride(1),
              packed.data_ptr(), packed.stride(0), packed.stride(1), bmax.data_ptr(), group_size,
              amp_lut.data_ptr(), cos_lut.data_ptr(), sin_lut.data_ptr(),
              out1.data_ptr(), out2.data_ptr(), out1.stride(0), out1.stride(1), M, N, K,
              _lib.ptr(ws), ws.numel() if ws is not None else 0, _lib.stream_handle(dev))
    return out1, out2


def dual_decode(packed, bmax, amp_lut, cos_lut, sin_lut, group_size=32):
    """FP16 decode of ``(K, N)`` int16 codes into ``(B1, B2)``, bit-exact with
    polar_kernels.py:64-79."""
    K, N = packed.shape
    dev = _lib.require_cuda(packed, bmax, amp_lut, cos_lut, sin_lut)
    amp_lut = _pad_table(amp_lut, 64)
    cos_lut = _pad_table(cos_lut, 1024)
    sin_lut = _pad_table(sin_lut, 1024)
    b1 = torch.empty((K, N), dtype=torch.float16, device=dev)
    b2 = torch.empty_like(b1)
    _lib.call("pp_dual_decode", packed.data_ptr(), packed.stride(0), packed.stride(1), K, N,
              bmax.contiguous().data_ptr(), group_size, amp_lut.data_ptr(), cos_lut.data_ptr(),
              sin_lut.data_ptr(), b1.data_ptr(), b2.data_ptr(), b1.stride(0), b1.stride(1),
              _lib.stream_handle(dev))
    return b1, b2
