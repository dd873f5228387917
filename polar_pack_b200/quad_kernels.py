"""Quad-pack (4 models, uint32 codes) -- drop-in for the reference ``quad_kernels.py``.

Same names, argument order, return types and error behaviour as the
reference module (quad_kernels.py:16-159); the decode + 4 matmuls run in
the hand-written sm_100a kernels of ``libpolarpack_b200.so``.

uint32 word: ``[norm 8][t1 8][t2 8][t3 8]``.
"""
from __future__ import annotations

import math

import torch

from . import _lib

MU = 255.0


def pack_quad_layer(w1, w2, w3, w4, mu=MU):
    """Pack 4 weight matrices ``(K, N)`` into uint32 codes + LUTs.

    Restates quad_kernels.py:16-50: per-model RMS ``s_k``, normalised
    4-vectors, ``r_max = 1.001 * max r``, mu-law norm and three angles
    quantised to 8 bits, seven FP16[256] tables.  Returns
    ``(codes uint32 (K,N), luts list[7] fp16, scales list[4] float)`` on the
    input device.  Layout producer, not on the timed path.
    """
    ws = [w1, w2, w3, w4]
    s = [torch.sqrt((w.float() ** 2).mean()) for w in ws]
    wn = [w.float() / sk for w, sk in zip(ws, s)]
    r = torch.sqrt(wn[0] ** 2 + wn[1] ** 2 + wn[2] ** 2 + wn[3] ** 2)
    r_max = float(r.max()) * 1.001
    log_mu = math.log1p(mu)
    t1 = torch.atan2(torch.sqrt(wn[1] ** 2 + wn[2] ** 2 + wn[3] ** 2), wn[0])
    t2 = torch.atan2(torch.sqrt(wn[2] ** 2 + wn[3] ** 2), wn[1])
    t3 = torch.atan2(wn[3], wn[2]) % (2 * math.pi)
    q = [torch.round(torch.log1p(mu * r / r_max) / log_mu * 255).clip(0, 255),
         torch.round(t1 / math.pi * 255).clip(0, 255),
         torch.round(t2 / math.pi * 255).clip(0, 255),
         torch.round(t3 / (2 * math.pi) * 255).clip(0, 255)]
    q = [x.to(torch.int64) for x in q]
    codes = ((q[0] << 24) | (q[1] << 16) | (q[2] << 8) | q[3]).to(torch.uint32)
    luts = [t.to(w1.device) for t in quad_luts(r_max, mu)]
    return codes, luts, [float(sk) for sk in s]


def quad_luts(r_max: float, mu: float = MU) -> list[torch.Tensor]:
    """The seven FP16[256] tables of quad_kernels.py:39-46 (float32 math, CPU)."""
    i = torch.arange(256, dtype=torch.float32)
    log_mu = math.log1p(mu)
    norm = ((torch.exp(i / 255 * log_mu) - 1) * r_max / mu).to(torch.float16)
    c12 = torch.cos(i / 255 * math.pi).to(torch.float16)
    s12 = torch.sin(i / 255 * math.pi).to(torch.float16)
    c3 = torch.cos(i / 255 * 2 * math.pi).to(torch.float16)
    s3 = torch.sin(i / 255 * 2 * math.pi).to(torch.float16)
    return [norm, c12, s12, c12.clone(), s12.clone(), c3, s3]


def _check_luts(luts, dev):
    if len(luts) != 7:
        raise ValueError("quad kernel takes 7 lookup tables")
    for t in luts:
        if t.dtype != torch.float16 or t.numel() < 256 or not t.is_contiguous():
            raise ValueError("lookup tables must be contiguous fp16 tensors of 256 entries")
        if t.device != dev:
            raise ValueError("lookup tables must be on the same device as the activations")


def _codes_u32(codes: torch.Tensor) -> torch.Tensor:
    if codes.dtype not in (torch.uint32, torch.int32):
        raise ValueError(f"codes must be uint32 (or an int32 view), got {codes.dtype}")
    return codes


def quad_bitpacked(a, codes, luts, scales):
    """``[out_k]_{k<4}``, ``out_k = fp16(s_k * (a @ W_k))`` in one pass over ``codes``.

    Drop-in for quad_kernels.py:146-159: ``a`` FP16 ``(M, K)``, ``codes``
    uint32 ``(K, N)`` with any strides, ``luts`` the seven FP16 tables,
    ``scales`` four floats.  Raises ``AssertionError`` on a K mismatch like
    the reference; launches on the current CUDA stream without syncing.
    """
    M, K = a.shape
    K_b, N = codes.shape
    assert K == K_b
    dev = _lib.require_cuda(a, codes)
    if a.dtype != torch.float16:
        raise ValueError("activations must be fp16")
    _check_luts(luts, dev)
    codes = _codes_u32(codes)
    outs = [torch.empty((M, N), dtype=torch.float16, device=dev) for _ in range(4)]
    lib = _lib.load()
    nbytes = _lib._size_t()
    _lib.check(lib.pp_quad_gemm_workspace_bytes(M, N, K, codes.stride(0), codes.stride(1),
                                                _lib.ctypes.byref(nbytes)))
    ws = _lib.workspace(dev, nbytes.value) if nbytes.value else None
    tables = _lib.cached_tables(luts, dev)   # replicated image, prepared once per table set
    _lib.call("pp_quad_gemm_prepared", a.data_ptr(), a.stride(0), a.stride(1),
              codes.data_ptr(), codes.stride(0), codes.stride(1),
              tables.data_ptr(), _lib.floats4(scales), _lib.ptrs(outs, 4),
              outs[0].stride(0), outs[0].stride(1), M, N, K,
              _lib.ptr(ws), ws.numel() if ws is not None else 0, _lib.stream_handle(dev))
    return outs


def quad_decode(codes, luts, scales=None):
    """FP16 decode of a ``(R, C)`` code matrix into four ``(R, C)`` FP16 matrices.

    Bit-exact with the reference kernel's chain (quad_kernels.py:103-121);
    with ``scales`` each result is multiplied by ``s_k`` in FP32 and rounded
    to FP16 once.
    """
    R, C = codes.shape
    dev = _lib.require_cuda(codes)
    _check_luts(luts, dev)
    codes = _codes_u32(codes)
    outs = [torch.empty((R, C), dtype=torch.float16, device=dev) for _ in range(4)]
    sc = None
    if scales is not None:
        sc = _lib.floats4(scales)
    _lib.call("pp_quad_decode", codes.data_ptr(), codes.stride(0), codes.stride(1), R, C,
              _lib.ptrs(luts, 7), _lib.ctypes.cast(sc, _lib.ctypes.c_void_p) if sc is not None else None,
              _lib.ptrs(outs, 4), outs[0].stride(0), outs[0].stride(1), _lib.stream_handle(dev))
    return outs
