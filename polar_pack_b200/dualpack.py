"""``.dualpack`` v2 streams on the GPU: reader, restore, Linear.

Format (reference polar_bitpack.py:26-29, 79-91, 160-172)::

    header '<8s I Q Q Q B B f I Q Q' (62 B): magic 'DUALPACK', version 2,
        n_pairs, n1, n2, amp_bits, phase_bits, mu, group_size, chunk_size, plug_n
    codes     2 B per pair, big-endian  amp << phase_bits | phase
    scales    fp16 group maxima; groups of group_size pairs restart at every
              chunk of chunk_size pairs
    plug_idx  uint32[plug_n]   ascending pair positions
    plug_val  fp16[plug_n]     exact amplitudes (the plug replaces the amplitude only)

:class:`DualPackDevice` keeps the stream in HBM as read.  :meth:`unpack`
restores both models' weights bit for bit as the reference's
``unpack_dual_models`` (polar_bitpack.py:194-260): the float64 tables are
computed here with numpy in the reference's order of operations and the GPU
repeats its float64 products.  :meth:`linear` serves one ``nn.Linear`` of the
pair straight from the file layout (``pp_dual_file_linear``).
"""
from __future__ import annotations

import ctypes
import math
import struct
from pathlib import Path

import numpy as np
import torch

from . import _lib
from .quadpack import unwrap_u32_positions, upload

MAGIC = b"DUALPACK"
VERSION = 2
HEADER_FMT = "<8s I Q Q Q B B f I Q Q"
HEADER_SIZE = struct.calcsize(HEADER_FMT)


class DualHeader:
    def __init__(self, buf):
        if len(buf) < HEADER_SIZE:
            raise ValueError("truncated .dualpack header")
        (magic, ver, self.n_pairs, self.n1, self.n2, self.amp_bits, self.phase_bits, self.mu, self.group_size,
         self.chunk_size, self.plug_n) = struct.unpack(HEADER_FMT, bytes(buf[:HEADER_SIZE]))
        if magic != MAGIC or ver != VERSION:
            raise ValueError(f"not a .dualpack v{VERSION} stream (magic={magic!r}, version={ver})")
        if self.amp_bits + self.phase_bits != 16 or not 1 <= self.phase_bits <= 15:
            raise ValueError("amp_bits + phase_bits must be 16")
        if self.group_size <= 0 or self.chunk_size <= 0:
            raise ValueError("group and chunk sizes must be positive")

    def n_groups(self) -> int:
        """Scales in the stream: groups restart at every chunk (polar_bitpack.py:201-203)."""
        ng = 0
        for s in range(0, self.n_pairs, self.chunk_size):
            ng += -(-min(self.chunk_size, self.n_pairs - s) // self.group_size)
        return ng


class DualPackFile:
    """Host view of a ``.dualpack`` stream (file path, bytes or numpy buffer)."""

    def __init__(self, src):
        if isinstance(src, (str, Path)):
            self.buf = np.memmap(str(src), dtype=np.uint8, mode="r")
        else:
            self.buf = np.frombuffer(src, dtype=np.uint8) if isinstance(src, (bytes, bytearray)) else src
        h = self.header = DualHeader(self.buf[:HEADER_SIZE])
        ng = h.n_groups()
        o = HEADER_SIZE
        self.codes = self.buf[o:o + 2 * h.n_pairs]
        o += 2 * h.n_pairs
        self.scales = self.buf[o:o + 2 * ng].view(np.float16)
        o += 2 * ng
        self.plug_idx = self.buf[o:o + 4 * h.plug_n].view(np.uint32)
        o += 4 * h.plug_n
        self.plug_vals = self.buf[o:o + 2 * h.plug_n].view(np.float16)
        o += 2 * h.plug_n
        if self.buf.size < o:
            raise ValueError(f"truncated .dualpack stream: {self.buf.size} bytes, header needs {o}")
        self.plug_pos = unwrap_u32_positions(np.asarray(self.plug_idx))
        if self.plug_pos.size and (np.any(np.diff(self.plug_pos) <= 0) or self.plug_pos[-1] >= h.n_pairs):
            raise ValueError("plug index is not strictly increasing inside [0, n_pairs)")

    def plug_range(self, start: int, stop: int) -> tuple[int, int]:
        return (int(np.searchsorted(self.plug_pos, start)), int(np.searchsorted(self.plug_pos, stop)))


def dual_tables(h: DualHeader) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """float64 ``amp_norm[a]``, ``cos(ang[ph])``, ``sin(ang[ph])`` computed as
    unpack_dual_models does (polar_bitpack.py:216-246)."""
    levels = 2 ** h.amp_bits - 1
    log_mu = np.log1p(h.mu)
    aq = np.arange(2 ** h.amp_bits, dtype=np.float64)
    amp = np.expm1(aq / levels * log_mu) / h.mu
    mask = (1 << h.phase_bits) - 1
    ang = np.arange(mask + 1).astype(np.float64) / (mask + 1) * 2 * np.pi - np.pi
    return amp, np.cos(ang), np.sin(ang)


class DualFileLinear:
    """One ``nn.Linear`` (out N, in K) of the two models, at pair ``offset``:
    ``(y1, y2) = (x W1^T, x W2^T)`` with ``W_j`` the FP16 restore."""

    def __init__(self, pack: "DualPackDevice", offset: int, N: int, K: int):
        self.pack, self.offset, self.N, self.K = pack, offset, N, K
        h, dev = pack.header, pack.device
        lo, hi = pack.file.plug_range(offset, offset + N * K)
        pos = torch.from_numpy(pack.file.plug_pos[lo:hi] - offset).to(dev)
        vals = torch.from_numpy(np.array(pack.file.plug_vals[lo:hi], copy=True)).to(dev)
        # exact FP16 weights of the plugged pairs: the plug amplitude with the
        # pair's phase, float64 products as in the restore
        bpos = (pos + offset) * 2
        hi_b = pack.codes[bpos].to(torch.int64)
        lo_b = pack.codes[bpos + 1].to(torch.int64)
        ph = ((hi_b << 8) | lo_b) & ((1 << h.phase_bits) - 1)
        amp = vals.float().double()
        w1 = (amp * pack.cos64[ph]).float().half()
        w2 = (amp * pack.sin64[ph]).float().half()
        self.plug_w = torch.stack([w1, w2], dim=1).contiguous()
        self.plug_col = (pos % K).to(torch.int32)
        rows = pos // K
        self.row_ptr = torch.searchsorted(rows, torch.arange(N + 1, device=dev)).to(torch.int32)
        # the plugged pairs' amplitude field cleared: they decode to zero and
        # enter through the plug list (the restore substitutes them itself)
        keep_hi = ((1 << h.phase_bits) - 1) >> 8
        pack.codes[bpos] = (hi_b & keep_hi).to(torch.uint8)
        if h.phase_bits < 8:
            pack.codes[bpos + 1] = (lo_b & ((1 << h.phase_bits) - 1)).to(torch.uint8)
        self._keep = (pos, vals)

    def __call__(self, x: torch.Tensor):
        if x.dim() != 2 or x.shape[1] != self.K or x.dtype != torch.float16:
            raise ValueError(f"x must be fp16 (M, {self.K})")
        dev = _lib.require_cuda(x)
        x = x.contiguous()
        M = x.shape[0]
        y = torch.empty((2, M, self.N), dtype=torch.float16, device=dev)
        pk, h = self.pack, self.pack.header
        for m0 in range(0, M, 4):
            m1 = min(M, m0 + 4)
            _lib.call("pp_dual_file_linear", pk.codes.data_ptr(), pk.scales.data_ptr(), h.chunk_size, h.group_size,
                      h.phase_bits, pk.amp32.data_ptr(), pk.cs32.data_ptr(), self.offset, self.row_ptr.data_ptr(),
                      self.plug_col.data_ptr(), self.plug_w.data_ptr(), x[m0:m1].data_ptr(), self.K, m1 - m0,
                      self.N, self.K, y[0, m0:].data_ptr(), y[1, m0:].data_ptr(), self.N, _lib.stream_handle(dev))
        return y[0], y[1]


class DualPackDevice:
    """The codes, scales and plug table of a ``.dualpack`` stream in HBM."""

    def __init__(self, f: DualPackFile, device):
        self.file, self.header, self.device = f, f.header, torch.device(device)
        h = self.header
        # codes padded to whole 16-byte words (the Linear reads 16-byte words)
        nb = -(-2 * h.n_pairs // 16) * 16
        self.codes = torch.zeros(max(nb, 16), dtype=torch.uint8, device=self.device)
        if h.n_pairs:
            self.codes[:2 * h.n_pairs] = upload(f.codes, np.uint8, self.device)
        self.scales = upload(f.scales, np.float16, self.device)
        self.plug_idx = upload(f.plug_idx, np.int32, self.device)
        self.plug_vals = upload(f.plug_vals, np.float16, self.device)
        amp, c, s = dual_tables(h)
        self.amp64 = torch.from_numpy(amp).to(self.device)
        self.cos64 = torch.from_numpy(c).to(self.device)
        self.sin64 = torch.from_numpy(s).to(self.device)
        self.amp32 = self.amp64.float()
        self.cs32 = torch.stack([self.cos64.float(), self.sin64.float()], dim=1).contiguous()
        self._linears: dict = {}

    def unpack(self, start: int = 0, stop: int | None = None, fp16: bool = False):
        """Both models' weights at pair positions ``[start, stop)``: float32
        (bit-exact with unpack_dual_models) or their FP16 roundings."""
        h = self.header
        stop = h.n_pairs if stop is None else stop
        n = stop - start
        dt = torch.float16 if fp16 else torch.float32
        w1 = torch.empty(n, dtype=dt, device=self.device)
        w2 = torch.empty(n, dtype=dt, device=self.device)
        lo, hi = self.file.plug_range(start, stop)
        ptr = lambda t, cond: t.data_ptr() if cond else None
        _lib.call("pp_dual_unpack", self.codes.data_ptr(), self.scales.data_ptr(), h.chunk_size, h.group_size,
                  h.phase_bits, self.amp64.data_ptr(), self.cos64.data_ptr(), self.sin64.data_ptr(),
                  self.plug_idx[lo:].data_ptr() if hi > lo else None,
                  self.plug_vals[lo:].data_ptr() if hi > lo else None, hi - lo,
                  ctypes.c_uint32(start & 0xFFFFFFFF), start, n, ptr(w1, not fp16), ptr(w2, not fp16),
                  ptr(w1, fp16), ptr(w2, fp16), _lib.stream_handle(self.device))
        return w1, w2

    def restore(self):
        """The two models as the reference restores them: ``w1[:n1]``, ``w2[:n2]``."""
        w1, w2 = self.unpack()
        return w1[:self.header.n1], w2[:self.header.n2]

    def linear(self, offset: int, N: int, K: int) -> DualFileLinear:
        """The Linear whose (N, K) weights start at pair ``offset`` (prepared once)."""
        if offset < 0 or N <= 0 or K <= 0 or offset + N * K > self.header.n_pairs:
            raise ValueError("Linear outside the stream")
        key = (offset, N, K)
        if key not in self._linears:
            self._linears[key] = DualFileLinear(self, offset, N, K)
        return self._linears[key]
