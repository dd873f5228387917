"""``.quadpack`` v2 streams on the GPU: reader, device upload, fused Linear.

Format (reference quaternion_packer.py:13-19, 93-132, 155-157)::

    header '<4sBBQBBBBfQ4ff4Q' (82 B): magic 'QUAD', version 2, n_models 4,
        n_min, bits (8, 8, 8, 8), mu, plug_n, rms s_0..s_3, r_max, tails_0..3
    codes     uint32[n_min]        word = nq<<24 | q1<<16 | q2<<8 | q3
    plug_idx  uint32[plug_n]       ascending flat positions
    plug_vals fp16[plug_n, 4]      RMS-normalised exact 4-tuples
    tail_k    fp16[tails_k]        raw weights of model k beyond n_min

Each ``nn.Linear`` of the packed models is an ``(out, in)`` row-major slice
of the flat stream, in the layer-map order of ``collect_weights``
(polar_main.py:25-51).  A :class:`QuadPackDevice` keeps codes and plug
values resident in HBM; :meth:`QuadPackDevice.linear` returns a
:class:`QuadLinearSlice` whose forward is one fused kernel launch
(``pp_quad_linear``) producing the four models' outputs.
"""
from __future__ import annotations

import ctypes
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np
import torch

from . import _lib
from .quad_kernels import quad_luts

MAGIC = b"QUAD"
VERSION = 2
N_MODELS = 4
MU = 255.0
HEADER_FMT = "<4sBBQBBBBfQ4ff4Q"
HEADER_SIZE = struct.calcsize(HEADER_FMT)


@dataclass
class QuadHeader:
    n: int
    plug_n: int
    scales: list
    r_max: float
    tails: list
    mu: float = MU
    bits: tuple = (8, 8, 8, 8)

    @classmethod
    def parse(cls, buf) -> "QuadHeader":
        if len(buf) < HEADER_SIZE:
            raise ValueError("truncated .quadpack header")
        h = struct.unpack(HEADER_FMT, bytes(buf[:HEADER_SIZE]))
        magic, ver, nm, n, nb, b1, b2, b3, mu, plug_n = h[:10]
        if magic != MAGIC or ver != VERSION:
            raise ValueError(f"not a .quadpack v{VERSION} stream (magic={magic!r}, version={ver})")
        if nm != N_MODELS or (nb, b1, b2, b3) != (8, 8, 8, 8):
            raise ValueError("only 4-model 8+8+8+8-bit .quadpack streams are defined")
        return cls(n=n, plug_n=plug_n, scales=list(h[10:14]), r_max=h[14], tails=list(h[15:19]),
                   mu=mu, bits=(nb, b1, b2, b3))

    def offsets(self) -> dict:
        codes = HEADER_SIZE
        plug_idx = codes + 4 * self.n
        plug_vals = plug_idx + 4 * self.plug_n
        tails = plug_vals + 8 * self.plug_n
        return dict(codes=codes, plug_idx=plug_idx, plug_vals=plug_vals, tails=tails,
                    end=tails + 2 * sum(self.tails))


def unwrap_u32_positions(idx_u32: np.ndarray) -> np.ndarray:
    """True int64 positions of an ascending plug index stored as uint32.

    The reference writes positions as uint32 (quaternion_packer.py:107);
    streams longer than 2^32 tuples wrap.  The true sequence is strictly
    increasing, so every decrease marks one more wrap.
    """
    x = idx_u32.astype(np.int64)
    if x.size < 2:
        return x
    wraps = np.concatenate([[0], np.cumsum(np.diff(x) < 0)])
    return x + (wraps.astype(np.int64) << 32)


class QuadPackFile:
    """Host view of a ``.quadpack`` stream (file path, bytes or numpy buffer)."""

    def __init__(self, src):
        if isinstance(src, (str, Path)):
            self.buf = np.memmap(str(src), dtype=np.uint8, mode="r")
        else:
            self.buf = np.frombuffer(src, dtype=np.uint8) if isinstance(src, (bytes, bytearray)) else src
        self.header = QuadHeader.parse(self.buf[:HEADER_SIZE])
        off = self.header.offsets()
        if self.buf.size < off["end"]:
            raise ValueError(f"truncated .quadpack stream: {self.buf.size} bytes, header needs {off['end']}")
        h = self.header
        self.codes = self.buf[off["codes"]:off["plug_idx"]].view(np.uint32)
        self.plug_idx = self.buf[off["plug_idx"]:off["plug_vals"]].view(np.uint32)
        self.plug_vals = self.buf[off["plug_vals"]:off["tails"]].view(np.float16).reshape(-1, 4)
        self.tails = []
        o = off["tails"]
        for t in h.tails:
            self.tails.append(self.buf[o:o + 2 * t].view(np.float16))
            o += 2 * t
        self.plug_pos = unwrap_u32_positions(np.asarray(self.plug_idx))
        if self.plug_pos.size and (np.any(np.diff(self.plug_pos) <= 0) or self.plug_pos[-1] >= h.n):
            raise ValueError("plug index is not strictly increasing inside [0, n)")

    def plug_range(self, start: int, stop: int) -> tuple[int, int]:
        """Slice ``[lo, hi)`` of the plug table covering flat positions ``[start, stop)``."""
        return (int(np.searchsorted(self.plug_pos, start)), int(np.searchsorted(self.plug_pos, stop)))


@dataclass
class QuadLinearSlice:
    """One packed ``nn.Linear`` (out=N, in=K) of a device-resident stream."""
    pack: "QuadPackDevice"
    offset: int
    N: int
    K: int
    p_lo: int
    p_hi: int
    codes: torch.Tensor
    plug_idx: torch.Tensor | None
    plug_vals: torch.Tensor | None
    plug_window_base: torch.Tensor | None
    # unit-major copy of the plug slice (pp_quad_prepare_unit_plugs): the
    # GEMV streams it beside the codes and needs no correction kernel
    unit_plugs: torch.Tensor | None = None
    unit_plug_off: torch.Tensor | None = None
    _ws: dict = field(default_factory=dict)

    @property
    def nbytes_stream(self) -> int:
        """Algorithmic bytes of one pass: codes + plug entries (index + values)."""
        return 4 * self.N * self.K + 12 * (self.p_hi - self.p_lo)

    def __call__(self, x: torch.Tensor, out=None) -> list[torch.Tensor]:
        return quad_linear(x, self, out=out)


class QuadPackDevice:
    """Codes, plug table and FP16 tables of a ``.quadpack`` stream resident on a GPU."""

    def __init__(self, f: QuadPackFile, device):
        self.file = f
        self.header = f.header
        self.device = torch.device(device)
        h = f.header
        self.codes = upload(f.codes, np.int32, self.device)
        self.plug_idx = upload(f.plug_idx, np.int32, self.device)
        self.plug_vals = upload(f.plug_vals, np.float16, self.device)
        # raw FP16 weights of each model beyond n_min (quaternion_packer.py:118-126)
        self.tails = [upload(t, np.float16, self.device) for t in f.tails]
        self.luts = [t.to(self.device) for t in quad_luts(h.r_max, MU)]
        # replicated shared-memory image of the tables, copied in by each launch
        self.tables = _lib.prepare_tables(self.luts, self.device)
        self.scales = [float(s) for s in h.scales]
        self._bad = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._linears: dict = {}

    def _plug_range(self, start: int, stop: int) -> tuple[int, int]:
        return self.file.plug_range(start, stop)

    def model_length(self, k: int) -> int:
        """Weights of model k: the coded range plus its FP16 tail."""
        return self.header.n + int(self.header.tails[k])

    def linear(self, offset: int, N: int, K: int):
        """The Linear whose ``(N, K)`` weights start at flat position ``offset``.

        A range inside the coded part ``[0, n_min)`` gives a
        :class:`QuadLinearSlice` (all four models, one fused launch).  A range
        that reaches past ``n_min`` gives a :class:`QuadTailedLinear`: its
        rows below ``n_min`` are served by the fused kernel, the rest from the
        FP16 tails of the models long enough to hold the whole Linear.

        The first call for a range prepares its plug entries in place (the
        norm byte of every plugged code of ``self.codes`` is zeroed, so it
        decodes to zeros and the plug value enters as a correction; see
        ``pp_quad_prepare_plugs``) and the slice is kept: later calls for the
        same range return it without preparing again.  :meth:`unpack` stays
        exact on prepared ranges because it substitutes every plugged
        position; a plain table decode of ``self.codes`` (``quad_decode``)
        does not and gives zeros at plugged positions.
        """
        n = self.header.n
        longest = max(self.model_length(k) for k in range(N_MODELS))
        if offset < 0 or N < 0 or K < 0 or offset + N * K > longest:
            raise ValueError(f"Linear [{offset}, {offset + N * K}) is outside every model (longest {longest})")
        key = (offset, N, K)
        hit = self._linears.get(key)
        if hit is None:
            if offset + N * K <= n:
                hit = self._make_linear(offset, N, K)
            else:
                hit = QuadTailedLinear(self, offset, N, K)
            self._linears[key] = hit
        return hit

    def _make_linear(self, offset: int, N: int, K: int) -> QuadLinearSlice:
        p_lo, p_hi = self._plug_range(offset, offset + N * K)
        codes = self.codes[offset:offset + N * K].view(N, K)
        if codes.data_ptr() % 16 and K % 4 == 0:
            # the streaming kernels read 16-byte aligned rows: a Linear at an
            # offset that is not a multiple of 4 codes gets its own aligned
            # copy, prepared instead of the stream's
            codes = codes.clone()
        pi = pv = wb = None
        if p_hi > p_lo:
            # one-time preparation: window index + zero norm byte of plugged codes
            wb = torch.empty(N * (-(-K // 64)) + 1, dtype=torch.int32, device=self.device)
            _lib.call("pp_quad_prepare_plugs", codes.data_ptr(), K, self.plug_idx.data_ptr(), p_lo, p_hi,
                      ctypes.c_uint32(offset & 0xFFFFFFFF), N, K, wb.data_ptr(), self._bad.data_ptr(),
                      _lib.stream_handle(self.device))
            pi = self.plug_idx[p_lo:p_hi]
            pv = self.plug_vals[p_lo:p_hi]
            up, uo = prepare_unit_plugs(pi, pv, wb, offset, N, K, self.device)
            return QuadLinearSlice(self, offset, N, K, p_lo, p_hi, codes, pi, pv, wb, up, uo)
        return QuadLinearSlice(self, offset, N, K, p_lo, p_hi, codes, pi, pv, wb)

    def check_plug_index(self) -> None:
        """Raise if any plug entry fell outside its Linear (syncs the device)."""
        bad = int(self._bad.item())
        if bad:
            raise ValueError(f"{bad} plug entries outside their Linear or out of order")

    def unpack(self, start: int = 0, stop: int | None = None, scaled: bool = True) -> list[torch.Tensor]:
        """GPU restore of flat positions ``[start, stop)`` into 4 FP16 vectors.

        FP16 table decode with plug substitution (quaternion_packer.py:170-196
        on the FP16 tables), optionally ``* s_k`` (one FP32 product, one FP16
        rounding).
        """
        stop = self.header.n if stop is None else stop
        n = stop - start
        outs = [torch.empty(n, dtype=torch.float16, device=self.device) for _ in range(4)]
        p_lo, p_hi = self._plug_range(start, stop)
        sc = _lib.floats4(self.scales) if scaled else None
        _lib.call("pp_quad_unpack", self.codes[start:].data_ptr() if n else self.codes.data_ptr(), n,
                  self.plug_idx.data_ptr(), self.plug_vals.data_ptr(), p_lo, p_hi,
                  ctypes.c_uint32(start & 0xFFFFFFFF), _lib.ptrs(self.luts, 7),
                  ctypes.cast(sc, ctypes.c_void_p) if sc is not None else None,
                  _lib.ptrs(outs, 4), _lib.stream_handle(self.device))
        return outs


@dataclass(frozen=True)
class TailSplit:
    """How a Linear at flat ``offset`` with ``(N, K)`` weights splits at ``n_min``.

    Rows ``[0, coded)`` lie wholly in the coded range; row ``coded`` is cut
    by ``n_min`` when ``straddle``; rows ``[first_tail, N)`` lie wholly past
    it, and their weights start ``tail_start`` elements into each model's
    tail.  ``present[k]``: model k is long enough to hold the whole Linear
    (quaternion_packer.py:55-57: model k has ``n_min + tails_k`` weights).
    """
    coded: int
    straddle: bool
    first_tail: int
    tail_start: int
    present: tuple


def tail_split(offset: int, N: int, K: int, n: int, tails) -> TailSplit:
    end = offset + N * K
    if offset >= n:
        coded, straddle = 0, False
    else:
        coded = min(N, (n - offset) // K) if K else N
        straddle = coded < N and offset + coded * K < n
    first = coded + (1 if straddle else 0)
    present = tuple(end <= n + int(t) for t in tails)
    return TailSplit(coded, straddle, first, offset + first * K - n, present)


class QuadTailedLinear:
    """A packed Linear whose flat range reaches past ``n_min``.

    The reference stores every weight of model k beyond the shortest model's
    length ``n_min`` as raw FP16 in that model's tail (quaternion_packer.py:
    118-126) and appends it unchanged when restoring (201-210).  Rows below
    ``n_min`` run on the fused quad kernel (all four models); the row cut by
    ``n_min`` is assembled once per model from its GPU-unpacked coded part
    (``fp16(w * s_k)``, plugs substituted) and its tail part; rows past
    ``n_min`` read each model's tail in place (``pp_f16_linear``).  A call
    returns four outputs ``(M, N)``; models whose weights end before the
    Linear does have no such Linear and get ``None``.
    """

    def __init__(self, pack: "QuadPackDevice", offset: int, N: int, K: int):
        h = pack.header
        self.pack, self.offset, self.N, self.K = pack, offset, N, K
        self.split = sp = tail_split(offset, N, K, h.n, h.tails)
        if not any(sp.present):
            raise ValueError(f"no model holds the Linear [{offset}, {offset + N * K})")
        self.coded = pack._make_linear(offset, sp.coded, K) if sp.coded else None
        self.straddle_rows = [None] * N_MODELS
        if sp.straddle:
            r0 = offset + sp.coded * K
            dec = pack.unpack(r0, h.n, scaled=True)
            for k in range(N_MODELS):
                if sp.present[k]:
                    row = torch.empty(K, dtype=torch.float16, device=pack.device)
                    row[:h.n - r0] = dec[k]
                    row[h.n - r0:] = pack.tails[k][:r0 + K - h.n]
                    self.straddle_rows[k] = row
        R = N - sp.first_tail
        self.tail_ptrs = [pack.tails[k][sp.tail_start:].data_ptr() if (sp.present[k] and R > 0) else None
                          for k in range(N_MODELS)]

    @property
    def present(self) -> tuple:
        return self.split.present

    def __call__(self, x: torch.Tensor, out=None) -> list:
        if x.dim() != 2 or x.shape[1] != self.K:
            raise ValueError(f"x must be (M, {self.K}), got {tuple(x.shape)}")
        if x.dtype != torch.float16:
            raise ValueError("x must be fp16")
        dev = _lib.require_cuda(x)
        if x.stride(1) != 1:
            x = x.contiguous()
        M, sp = x.shape[0], self.split
        if out is None:
            buf = torch.empty((N_MODELS, M, self.N), dtype=torch.float16, device=dev)
            out = [buf[k] for k in range(N_MODELS)]
        if self.coded is not None:
            quad_linear(x, self.coded, out=[o[:, :sp.coded] for o in out])
        lib, s = _lib.load(), _lib.stream_handle(dev)
        if sp.straddle:
            w = (ctypes.c_void_p * 4)(*[_lib.ptr(r) for r in self.straddle_rows])
            o = _lib.ptrs([o_[:, sp.coded:] for o_ in out], 4)
            _lib.check(lib.pp_f16_linear(x.data_ptr(), x.stride(0), 0, M, self.K, w, self.K, 1, o,
                                         out[0].stride(0), out[0].stride(1), s))
        R = self.N - sp.first_tail
        if R > 0:
            w = (ctypes.c_void_p * 4)(*self.tail_ptrs)
            o = _lib.ptrs([o_[:, sp.first_tail:] for o_ in out], 4)
            _lib.check(lib.pp_f16_linear(x.data_ptr(), x.stride(0), 0, M, self.K, w, self.K, R, o,
                                         out[0].stride(0), out[0].stride(1), s))
        return [out[k] if sp.present[k] else None for k in range(N_MODELS)]


def upload(arr, view_dtype, device, chunk: int = 1 << 26) -> torch.Tensor:
    """Copy a host array (read-only memmaps included) to ``device`` in
    chunks, viewed as ``view_dtype``; each chunk is copied into a writable
    host buffer first, so no tensor ever aliases read-only memory."""
    a = np.asarray(arr).view(view_dtype)
    out = torch.empty(a.shape, dtype=torch.from_numpy(np.empty(0, view_dtype)).dtype, device=device)
    flat_in, flat_out = a.reshape(-1), out.view(-1)
    for i in range(0, flat_in.size, chunk):
        j = min(i + chunk, flat_in.size)
        flat_out[i:j].copy_(torch.from_numpy(np.array(flat_in[i:j], copy=True)))
    return out


def prepare_unit_plugs(plug_idx: torch.Tensor, plug_vals: torch.Tensor, window_base: torch.Tensor, offset: int,
                       N: int, K: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """Unit-major plug stream and its unit offsets for one Linear's plug slice."""
    nbytes, noff = _lib._size_t(), ctypes.c_int64()
    P = int(plug_idx.numel())
    _lib.check(_lib.load().pp_quad_unit_plugs_bytes(N, K, P, ctypes.byref(nbytes), ctypes.byref(noff)))
    stream = torch.empty(max(nbytes.value, 16), dtype=torch.uint8, device=device)
    off = torch.empty(noff.value, dtype=torch.int32, device=device)
    _lib.call("pp_quad_prepare_unit_plugs", _lib.ptr(plug_idx), _lib.ptr(plug_vals), P,
              ctypes.c_uint32(offset & 0xFFFFFFFF), window_base.data_ptr(), N, K, stream.data_ptr(),
              stream.numel(), off.data_ptr(), _lib.stream_handle(torch.device(device)))
    return stream, off


def quad_linear_workspace_bytes(M: int, N: int, K: int) -> int:
    nbytes = _lib._size_t()
    _lib.check(_lib.load().pp_quad_linear_workspace_bytes(M, N, K, ctypes.byref(nbytes)))
    return nbytes.value


def quad_linear(x: torch.Tensor, layer: QuadLinearSlice, out=None) -> list[torch.Tensor]:
    """``[y_k]``, ``y_k = fp16(s_k * x @ Wp_k^T)`` for one packed Linear.

    ``x`` is FP16 ``(M, K)`` (any strides).  ``Wp_k`` is the FP16 decode with
    plug values substituted; one kernel launch streams the codes once.  The
    per-Linear C arguments are built once and kept on the slice, so a call
    costs one output allocation and one library call.
    """
    if x.dim() != 2 or x.shape[1] != layer.K:
        raise ValueError(f"x must be (M, {layer.K}), got {tuple(x.shape)}")
    if x.dtype != torch.float16:
        raise ValueError("x must be fp16")
    dev = _lib.require_cuda(x, layer.codes)
    if x.stride(1) != 1 or x.data_ptr() % 8 or (x.stride(0) * 2) % 8:
        x = x.contiguous() if x.stride(1) != 1 else x.clone()  # the kernel reads 8-byte activation groups
    M = x.shape[0]
    if out is None:
        buf = torch.empty((4, M, layer.N), dtype=torch.float16, device=dev)
        out = [buf[0], buf[1], buf[2], buf[3]]
    c = layer._ws.get("args")
    if c is None:
        pk = layer.pack
        lib = _lib.load()
        head = (layer.codes.data_ptr(), layer.K, _lib.ptr(layer.plug_idx), _lib.ptr(layer.plug_vals),
                _lib.ptr(layer.plug_window_base), ctypes.c_uint32(layer.offset & 0xFFFFFFFF))
        if layer.unit_plugs is not None:
            c = (lib.pp_quad_linear_fused, *head, layer.unit_plugs.data_ptr(), layer.unit_plug_off.data_ptr(),
                 pk.tables.data_ptr(), _lib.floats4(pk.scales))
        else:
            c = (lib.pp_quad_linear_prepared, *head, pk.tables.data_ptr(), _lib.floats4(pk.scales))
        layer._ws["args"] = c
    nb = layer._ws.get(("ws", M))
    if nb is None:
        nb = layer._ws[("ws", M)] = quad_linear_workspace_bytes(M, layer.N, layer.K)
    ws = _lib.workspace(dev, nb) if nb else None
    _lib.check(c[0](x.data_ptr(), x.stride(0), x.stride(1), *c[1:],
                    _lib.ptrs(out, 4), out[0].stride(0), out[0].stride(1), M, layer.N, layer.K,
                    _lib.ptr(ws), ws.numel() if ws is not None else 0, _lib.stream_handle(dev)))
    return out


def linear_desc(x: torch.Tensor, layer: QuadLinearSlice, out, per_model_x: bool = False, bias=None,
                resid=None, x_il: torch.Tensor | None = None) -> "_lib.QuadLinearDesc":
    """The C descriptor of one ``quad_linear(x, layer, out)`` (pointers of the
    given tensors: keep them alive while the descriptor is used).

    ``per_model_x``: ``x`` has four rows, model k multiplies row k and writes
    row 0 of ``out[k]``; ``x_il`` (optional) holds the same rows interleaved,
    ``x_il[4 i + k] = x[k][i]``, which the fused plug correction reads with
    one load per plugged column.  ``bias`` / ``resid``: four FP16 vectors (or
    None) of the epilogue ``fp16(s_k acc + bias_k)``, then ``+ resid_k``
    (``resid`` indexed like ``out``; it may be ``out`` itself)."""
    d = _lib.QuadLinearDesc()
    d.flags = _lib.PER_MODEL_X if per_model_x else 0
    if x_il is not None:
        if not per_model_x or x_il.numel() < 4 * layer.K or x_il.dtype != torch.float16:
            raise ValueError("x_il: per-model activations only, FP16, 4 * K values")
        d.x_il = x_il.data_ptr()
    for k in range(4):
        d.bias[k] = bias[k].data_ptr() if bias is not None and bias[k] is not None else None
        d.resid[k] = resid[k].data_ptr() if resid is not None and resid[k] is not None else None
    d.x, d.ldx_m, d.ldx_k = x.data_ptr(), x.stride(0), x.stride(1)
    d.codes, d.ldw = layer.codes.data_ptr(), layer.codes.stride(0)
    d.plug_idx, d.plug_vals = _lib.ptr(layer.plug_idx), _lib.ptr(layer.plug_vals)
    d.plug_window_base, d.base_lo32 = _lib.ptr(layer.plug_window_base), layer.offset & 0xFFFFFFFF
    d.unit_plugs, d.unit_plug_off = _lib.ptr(layer.unit_plugs), _lib.ptr(layer.unit_plug_off)
    d.tables = layer.pack.tables.data_ptr()
    for k in range(4):
        d.scales[k] = float(layer.pack.scales[k])
        d.out[k] = out[k].data_ptr() if out is not None else None
    # output strides (gathered members write no out[], but a residual is read with these strides)
    src = out if out is not None else resid
    d.ldo_m, d.ldo_n = (src[0].stride(0), src[0].stride(1)) if src is not None else (0, 1)
    d.M, d.N, d.K = (1 if per_model_x else x.shape[0]), layer.N, layer.K
    return d


class QuadLinearGroup:
    """Independent packed Linears launched together (``pp_quad_linear_group``).

    ``layers[j]`` reads ``xs[j]`` and writes ``outs[j]`` (four ``(M, N_j)``
    tensors); the tensors are fixed at construction, so a call is one library
    call (and one kernel launch when every member is a batch-1 Linear with
    unit plugs -- ``single_launch``), and it can be captured in a CUDA graph.
    The members must not read each other's outputs.
    """

    def __init__(self, layers, xs, outs, per_model_x: bool = False, biases=None, resids=None, x_ils=None):
        if not (len(layers) == len(xs) == len(outs)) or not layers:
            raise ValueError("one input and one output set per Linear")
        for x, l in zip(xs, layers):
            if x.dim() != 2 or x.shape[1] != l.K or x.dtype != torch.float16:
                raise ValueError("each x must be fp16 (M, K) of its Linear")
            if per_model_x and x.shape[0] != 4:
                raise ValueError("per-model activations: x must have one row per model (4)")
        self.layers, self.xs, self.outs = list(layers), list(xs), [list(o) for o in outs]
        self.device = _lib.require_cuda(*self.xs)
        n = len(layers)
        biases = biases or [None] * n
        resids = resids or [None] * n
        x_ils = x_ils or [None] * n
        self._keep = (biases, resids, x_ils)
        self.descs = (_lib.QuadLinearDesc * n)(*[linear_desc(x, l, o, per_model_x, b, r, xi)
                                                 for x, l, o, b, r, xi in zip(xs, layers, outs, biases, resids,
                                                                              x_ils)])
        lib = _lib.load()
        nb = _lib._size_t()
        _lib.check(lib.pp_quad_linear_group_workspace_bytes(n, self.descs, ctypes.byref(nb)))
        self.ws = torch.zeros(max(nb.value, 256), dtype=torch.uint8, device=self.device)
        self.single_launch = bool(lib.pp_quad_linear_group_single_launch(n, self.descs))
        self._lib = lib

    def __call__(self, stream=None):
        s = stream if stream is not None else _lib.stream_handle(self.device)
        rc = self._lib.pp_quad_linear_group(len(self.layers), self.descs, self.ws.data_ptr(), self.ws.numel(), s)
        if rc:
            _lib.check(rc)
        return self.outs


def layer_offsets(layer_map: list[dict]) -> list[tuple[str, int, tuple[int, int]]]:
    """``(name, flat offset, (out, in))`` per entry of a ``collect_weights`` layer map.

    The offset is the running sum of ``numel`` in map order, as
    ``replace_model_weights`` walks it (polar_packer.py:296-316).
    """
    res, off = [], 0
    for e in layer_map:
        shape = tuple(int(s) for s in e["shape"])
        res.append((e["name"], off, shape))
        off += int(e["numel"])
    return res


# ------------------------------------------------------------ GPU packer --
def _quantize_chunk_torch(wc, r_max: float, with_err: bool):
    """Codes (and relative decode error) of one chunk; quaternion_packer.py:30-49.

    Codes come from float32 math on the normalised weights; the error uses
    float64 like the reference's ``thr_collect`` branch.
    """
    import math
    w1, w2, w3, w4 = wc
    r = torch.sqrt(w1 * w1 + w2 * w2 + w3 * w3 + w4 * w4)
    t1 = torch.atan2(torch.sqrt(w2 * w2 + w3 * w3 + w4 * w4), w1)
    t2 = torch.atan2(torch.sqrt(w3 * w3 + w4 * w4), w2)
    t3 = torch.remainder(torch.atan2(w4, w3), 2 * math.pi)
    log_mu = math.log1p(MU)
    nq = torch.round(torch.log1p(MU * r / r_max) / log_mu * 255).clamp(0, 255).to(torch.int64)
    q1 = torch.round(t1 / math.pi * 255).clamp(0, 255).to(torch.int64)
    q2 = torch.round(t2 / math.pi * 255).clamp(0, 255).to(torch.int64)
    q3 = torch.round(t3 / (2 * math.pi) * 255).clamp(0, 255).to(torch.int64)
    codes = ((nq << 24) | (q1 << 16) | (q2 << 8) | q3).to(torch.uint32)
    if not with_err:
        return codes, None
    rr = (torch.exp(nq.double() / 255 * log_mu) - 1) * r_max / MU
    a1, a2, a3 = q1.double() / 255 * math.pi, q2.double() / 255 * math.pi, q3.double() / 255 * 2 * math.pi
    s1, s2 = torch.sin(a1), torch.sin(a2)
    rw = (rr * torch.cos(a1), rr * s1 * torch.cos(a2), rr * s1 * s2 * torch.cos(a3), rr * s1 * s2 * torch.sin(a3))
    err = torch.sqrt(sum((wc[k].double() - rw[k]) ** 2 for k in range(4))) / torch.clamp(r.double(), min=1e-12)
    return codes, err


def pack_quad_device(models, plug_cap: float = 0.05, seed: int = 42, windows: int = 100,
                     window: int = 1_000_000, chunk: int = 1 << 24) -> dict:
    """Pack four 1-D weight tensors into ``.quadpack`` v2 sections on their device.

    Restates pack_quad (quaternion_packer.py:52-138): pass A float64 RMS on
    the common length, pass B ``r_max * 1.001`` and the ``(1 - plug_cap)``
    percentile of the decode error over ``windows`` random windows drawn with
    numpy's ``default_rng(seed)``, pass C codes and plug entries (ascending
    positions, FP16 normalised 4-tuples), then raw FP16 tails.  Returns a
    dict of device tensors plus header fields; :func:`to_bytes` serialises
    it.  Transcendentals run on the GPU, so a code can differ from the numpy
    writer's by one step where a value sits on a rounding boundary.
    """
    dev = models[0].device
    lengths = [int(m.numel()) for m in models]
    n = min(lengths)
    tails = [L - n for L in lengths]
    s = [float(torch.sqrt((m[:n].double() ** 2).sum() / n)) for m in models]
    r_max = 0.0
    for i in range(0, n, chunk):
        wc = [m[i:min(i + chunk, n)].float() / sk for m, sk in zip(models, s)]
        r_max = max(r_max, float(torch.sqrt(sum(x * x for x in wc)).max()))
    r_max *= 1.001
    window = min(window, max(1, n - 1))
    rng = np.random.default_rng(seed)
    starts = rng.integers(0, max(1, n - window), windows)
    errs = []
    for st in starts:
        wc = [m[st:st + window].float() / sk for m, sk in zip(models, s)]
        errs.append(_quantize_chunk_torch(wc, r_max, True)[1].cpu().numpy())
    thr = float(np.percentile(np.concatenate(errs), (1 - plug_cap) * 100))
    codes = torch.empty(n, dtype=torch.uint32, device=dev)
    pidx, pval = [], []
    for i in range(0, n, chunk):
        wc = [m[i:min(i + chunk, n)].float() / sk for m, sk in zip(models, s)]
        c, err = _quantize_chunk_torch(wc, r_max, True)
        codes[i:i + c.numel()] = c
        mask = err > thr
        idx = torch.nonzero(mask).flatten()
        if idx.numel():
            pidx.append(idx + i)
            pval.append(torch.stack([w[idx] for w in wc], dim=1).half())
    plug_idx = torch.cat(pidx) if pidx else torch.zeros(0, dtype=torch.int64, device=dev)
    plug_vals = torch.cat(pval) if pval else torch.zeros((0, 4), dtype=torch.float16, device=dev)
    tail_t = [m[n:].half() for m in models]
    return dict(n=n, scales=s, r_max=r_max, tails=tails, codes=codes, plug_pos=plug_idx,
                plug_vals=plug_vals, tail_vals=tail_t, threshold=thr)


def pack_quad_generated(gen, n: int, plug_cap: float = 0.05, seed: int = 42, windows: int = 100,
                        window: int = 1_000_000, chunk: int = 1 << 24, device=None) -> dict:
    """:func:`pack_quad_device` for models too large to hold at once.

    ``gen(start, stop)`` returns the four models' weights at flat positions
    ``[start, stop)`` (four 1-D tensors on ``device``), the same values for a
    position whatever range asks for it.  The passes are those of pack_quad
    (quaternion_packer.py:52-138): float64 RMS, r_max and the plug threshold
    over seeded windows, then codes and plug entries chunk by chunk, so only
    the codes and one chunk live on the device.  Models of equal length (no
    tails).
    """
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    acc = torch.zeros(4, dtype=torch.float64, device=dev)
    r_max = torch.zeros((), dtype=torch.float32, device=dev)
    for i in range(0, n, chunk):
        ws = gen(i, min(i + chunk, n))
        for k, w in enumerate(ws):
            acc[k] += (w.double() ** 2).sum()
    s = [float(torch.sqrt(acc[k] / n)) for k in range(4)]
    for i in range(0, n, chunk):
        wc = [w.float() / sk for w, sk in zip(gen(i, min(i + chunk, n)), s)]
        r_max = torch.maximum(r_max, torch.sqrt(sum(x * x for x in wc)).max())
    r_max = float(r_max) * 1.001
    window = min(window, max(1, n - 1))
    rng = np.random.default_rng(seed)
    starts = rng.integers(0, max(1, n - window), windows)
    errs = []
    for st in starts:
        wc = [w.float() / sk for w, sk in zip(gen(int(st), int(st) + window), s)]
        errs.append(_quantize_chunk_torch(wc, r_max, True)[1].cpu().numpy())
    thr = float(np.percentile(np.concatenate(errs), (1 - plug_cap) * 100))
    codes = torch.empty(n, dtype=torch.uint32, device=dev)
    pidx, pval = [], []
    for i in range(0, n, chunk):
        wc = [w.float() / sk for w, sk in zip(gen(i, min(i + chunk, n)), s)]
        c, err = _quantize_chunk_torch(wc, r_max, True)
        codes[i:i + c.numel()] = c
        idx = torch.nonzero(err > thr).flatten()
        if idx.numel():
            pidx.append(idx + i)
            pval.append(torch.stack([w[idx] for w in wc], dim=1).half())
    plug_idx = torch.cat(pidx) if pidx else torch.zeros(0, dtype=torch.int64, device=dev)
    plug_vals = torch.cat(pval) if pval else torch.zeros((0, 4), dtype=torch.float16, device=dev)
    empty = torch.zeros(0, dtype=torch.float16, device=dev)
    return dict(n=n, scales=s, r_max=r_max, tails=[0, 0, 0, 0], codes=codes, plug_pos=plug_idx,
                plug_vals=plug_vals, tail_vals=[empty] * 4, threshold=thr)


class SyntheticModels:
    """Four correlated FP16 weight streams of any length, generated on demand:
    base N(0, 0.02) + per-model delta N(0, 0.002), 0.1% of entries x 20 (the
    benchmark distribution).  Blocks of ``block`` positions have their own
    seeds, so ``self(start, stop)`` gives the same values for a position
    whatever range is asked for (what :func:`pack_quad_generated` needs)."""

    def __init__(self, seed: int, device, block: int = 1 << 20):
        self.seed, self.device, self.block = seed, torch.device(device), block

    def _block(self, b: int) -> list[torch.Tensor]:
        g = torch.Generator(device=self.device)
        g.manual_seed(self.seed * 1_000_003 + b)
        B = self.block
        base = torch.randn(B, generator=g, device=self.device) * 0.02
        out = []
        for _ in range(4):
            w = base + torch.randn(B, generator=g, device=self.device) * 0.002
            w = torch.where(torch.rand(B, generator=g, device=self.device) < 0.001, w * 20, w)
            out.append(w.half())
        return out

    def __call__(self, start: int, stop: int) -> list[torch.Tensor]:
        B = self.block
        b0, b1 = start // B, (stop + B - 1) // B
        parts = [self._block(b) for b in range(b0, b1)]
        res = []
        for k in range(4):
            cat = torch.cat([p[k] for p in parts]) if len(parts) > 1 else parts[0][k]
            res.append(cat[start - b0 * B:stop - b0 * B])
        return res


def to_bytes(p: dict) -> bytes:
    """Serialise :func:`pack_quad_device` output as a ``.quadpack`` v2 stream."""
    hdr = struct.pack(HEADER_FMT, MAGIC, VERSION, N_MODELS, p["n"], 8, 8, 8, 8, MU,
                      int(p["plug_pos"].numel()), *p["scales"], p["r_max"], *p["tails"])
    parts = [hdr, p["codes"].cpu().numpy().tobytes(),
             (p["plug_pos"].cpu().numpy() & 0xFFFFFFFF).astype(np.uint32).tobytes(),
             p["plug_vals"].cpu().numpy().tobytes()]
    parts += [t.cpu().numpy().tobytes() for t in p["tail_vals"] if t.numel()]
    return b"".join(parts)


class DevicePackedStream(QuadPackDevice):
    """A :class:`QuadPackDevice` built from :func:`pack_quad_device` output
    without a host round trip (used for synthetic full-size streams)."""

    def __init__(self, p: dict):
        self.file = None
        self.device = p["codes"].device
        self.header = QuadHeader(n=p["n"], plug_n=int(p["plug_pos"].numel()), scales=list(p["scales"]),
                                 r_max=p["r_max"], tails=list(p["tails"]))
        self.codes = p["codes"]
        pos = p["plug_pos"].to(torch.int64)
        self._pos_host = pos.cpu().numpy()
        self.plug_idx = (pos & 0xFFFFFFFF).to(torch.int64).to(torch.int32) if pos.numel() else \
            torch.zeros(0, dtype=torch.int32, device=self.device)
        self.plug_vals = p["plug_vals"].contiguous()
        self.tails = [t.contiguous() for t in p["tail_vals"]]
        self.luts = [t.to(self.device) for t in quad_luts(p["r_max"], MU)]
        self.tables = _lib.prepare_tables(self.luts, self.device)
        self.scales = [float(x) for x in p["scales"]]
        self._bad = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._linears = {}

    def _plug_range(self, start: int, stop: int) -> tuple[int, int]:
        return (int(np.searchsorted(self._pos_host, start)), int(np.searchsorted(self._pos_host, stop)))
