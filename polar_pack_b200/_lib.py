"""ctypes binding of the in-tree CUDA library ``libpolarpack_b200.so``.

The library exposes a plain C ABI (``include/polar_pack_b200.h``); this
module declares the argument types, loads it once, and turns non-zero status
codes into Python exceptions.  There is no fallback: if the shared object is
missing or fails to load, every call raises ``RuntimeError``.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libpolarpack_b200.so"

PP_OK, PP_ERR_INVALID, PP_ERR_WORKSPACE, PP_ERR_CUDA = 0, 1, 2, 3

_c_void_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_u32 = ctypes.c_uint32
_size_t = ctypes.c_size_t
_int = ctypes.c_int
_PTR7 = _c_void_p * 7
_PTR4 = _c_void_p * 4
_F4 = ctypes.c_float * 4

class QuadLinearDesc(ctypes.Structure):
    """``pp_quad_linear_desc``: one member of a grouped launch."""
    _fields_ = [("x", ctypes.c_void_p), ("ldx_m", ctypes.c_int64), ("ldx_k", ctypes.c_int64),
                ("codes", ctypes.c_void_p), ("ldw", ctypes.c_int64),
                ("plug_idx", ctypes.c_void_p), ("plug_vals", ctypes.c_void_p),
                ("plug_window_base", ctypes.c_void_p), ("base_lo32", ctypes.c_uint32),
                ("unit_plugs", ctypes.c_void_p), ("unit_plug_off", ctypes.c_void_p),
                ("tables", ctypes.c_void_p), ("scales", ctypes.c_float * 4),
                ("out", ctypes.c_void_p * 4), ("ldo_m", ctypes.c_int64), ("ldo_n", ctypes.c_int64),
                ("M", ctypes.c_int64), ("N", ctypes.c_int64), ("K", ctypes.c_int64),
                ("flags", ctypes.c_uint32), ("bias", ctypes.c_void_p * 4), ("resid", ctypes.c_void_p * 4),
                ("x_il", ctypes.c_void_p)]

PER_MODEL_X = 1


_DESC_P = ctypes.POINTER(QuadLinearDesc)

_SIGNATURES = {
    "pp_last_error": ([], ctypes.c_char_p),
    "pp_version": ([], _int),
    "pp_device_sm_count": ([_int], _int),
    "pp_set_launch_overlap": ([_int], _int),
    "pp_quad_gemm_workspace_bytes": ([_i64, _i64, _i64, _i64, _i64, ctypes.POINTER(_size_t)], _int),
    "pp_quad_gemm": ([_c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _PTR7, _F4, _PTR4, _i64, _i64,
                      _i64, _i64, _i64, _c_void_p, _size_t, _c_void_p], _int),
    "pp_quad_gemm_static_scratch": ([_c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _PTR7, _F4, _PTR4, _i64,
                                     _i64, _i64, _i64, _i64, _c_void_p], _int),
    "pp_quad_tables_bytes": ([ctypes.POINTER(_size_t)], _int),
    "pp_quad_prepare_tables": ([_PTR7, _c_void_p, _c_void_p], _int),
    "pp_quad_gemm_prepared": ([_c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _c_void_p, _F4, _PTR4, _i64, _i64,
                               _i64, _i64, _i64, _c_void_p, _size_t, _c_void_p], _int),
    "pp_quad_linear_prepared": ([_c_void_p, _i64, _i64, _c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p, _u32,
                                 _c_void_p, _F4, _PTR4, _i64, _i64, _i64, _i64, _i64, _c_void_p, _size_t,
                                 _c_void_p], _int),
    "pp_quad_linear_workspace_bytes": ([_i64, _i64, _i64, ctypes.POINTER(_size_t)], _int),
    "pp_quad_linear": ([_c_void_p, _i64, _i64, _c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p, _u32,
                        _PTR7, _F4, _PTR4, _i64, _i64, _i64, _i64, _i64, _c_void_p, _size_t,
                        _c_void_p], _int),
    "pp_quad_prepare_plugs": ([_c_void_p, _i64, _c_void_p, _i64, _i64, _u32, _i64, _i64, _c_void_p,
                               _c_void_p, _c_void_p], _int),
    "pp_quad_unit_plugs_bytes": ([_i64, _i64, _i64, ctypes.POINTER(_size_t), ctypes.POINTER(_i64)], _int),
    "pp_quad_prepare_unit_plugs": ([_c_void_p, _c_void_p, _i64, _u32, _c_void_p, _i64, _i64, _c_void_p, _size_t,
                                    _c_void_p, _c_void_p], _int),
    "pp_quad_linear_fused": ([_c_void_p, _i64, _i64, _c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p, _u32,
                              _c_void_p, _c_void_p, _c_void_p, _F4, _PTR4, _i64, _i64, _i64, _i64, _i64,
                              _c_void_p, _size_t, _c_void_p], _int),
    "pp_quad_linear_group_workspace_bytes": ([_int, _DESC_P, ctypes.POINTER(_size_t)], _int),
    "pp_quad_linear_group_single_launch": ([_int, _DESC_P], _int),
    "pp_quad_linear_group": ([_int, _DESC_P, _c_void_p, _size_t, _c_void_p], _int),
    "pp_quad_linear_group_gather": ([_int, _DESC_P, _int, _c_void_p, _i64, ctypes.POINTER(_i64), _c_void_p,
                                     _c_void_p, _c_void_p, _size_t, _c_void_p], _int),
    "pp_ipc_handle": ([_c_void_p, _c_void_p, ctypes.POINTER(_size_t)], _int),
    "pp_ipc_open": ([_c_void_p, ctypes.POINTER(_c_void_p)], _int),
    "pp_ipc_close": ([_c_void_p], _int),
    "pp_quad_linear_gather": ([_c_void_p, _i64, _c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p, _u32,
                               _c_void_p, _c_void_p, _c_void_p, _F4, _int, _c_void_p, _i64, _i64, _c_void_p,
                               _c_void_p, _i64, _i64, _c_void_p, _size_t, _c_void_p], _int),
    "pp_gather_wait": ([_c_void_p, _int, _c_void_p, _c_void_p, _c_void_p], _int),
    "pp_quad_decode": ([_c_void_p, _i64, _i64, _i64, _i64, _PTR7, _c_void_p, _PTR4, _i64, _i64,
                        _c_void_p], _int),
    "pp_quad_unpack": ([_c_void_p, _i64, _c_void_p, _c_void_p, _i64, _i64, _u32, _PTR7, _c_void_p,
                        _PTR4, _c_void_p], _int),
    "pp_f16_linear": ([_c_void_p, _i64, _i64, _i64, _i64, _PTR4, _i64, _i64, _PTR4, _i64, _i64, _c_void_p], _int),
    "pp_embed_rows": ([_c_void_p, _PTR4, _i64, _i64, _c_void_p, _i64, _c_void_p, _c_void_p], _int),
    "pp_rmsnorm_rows": ([_c_void_p, _i64, _PTR4, _i64, ctypes.c_float, _c_void_p, _i64, _c_void_p, _c_void_p, _int,
                         _c_void_p, _c_void_p, _c_void_p], _int),
    "pp_decode_attention_workspace_bytes": ([_i64, _i64, _i64, ctypes.POINTER(_size_t)], _int),
    "pp_decode_attention": ([_c_void_p, _i64, _i64, _i64, _i64, _c_void_p, _c_void_p, _PTR4, _PTR4, _i64,
                             _c_void_p, ctypes.c_float, _c_void_p, _i64, _c_void_p, _i64, _c_void_p, _size_t,
                             _c_void_p, _c_void_p, _int, _c_void_p, _c_void_p, _c_void_p], _int),
    "pp_swiglu_rows": ([_c_void_p, _i64, _i64, _c_void_p, _i64, _c_void_p, _c_void_p, _int, _c_void_p, _c_void_p,
                        _c_void_p], _int),
    "pp_dual_gemm_workspace_bytes": ([_i64, _i64, _i64, _i64, _i64, ctypes.POINTER(_size_t)], _int),
    "pp_dual_gemm": ([_c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _c_void_p, _i64, _c_void_p,
                      _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _i64, _i64,
                      _c_void_p, _size_t, _c_void_p], _int),
    "pp_dual_unpack": ([_c_void_p, _c_void_p, _i64, _i64, _int, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                        _c_void_p, _i64, _u32, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p],
                       _int),
    "pp_dual_file_linear": ([_c_void_p, _c_void_p, _i64, _i64, _int, _c_void_p, _c_void_p, _i64, _c_void_p,
                             _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _i64, _c_void_p, _c_void_p, _i64,
                             _c_void_p], _int),
    "pp_dual_decode": ([_c_void_p, _i64, _i64, _i64, _i64, _c_void_p, _i64, _c_void_p, _c_void_p,
                        _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _c_void_p], _int),
}

_lock = threading.Lock()
_lib = None


def exported_symbols() -> list[str]:
    """Every entry point the header declares (and this module binds)."""
    return list(_SIGNATURES)


def load() -> ctypes.CDLL:
    """Load the shared library (once) and declare every signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = Path(os.environ.get("POLAR_PACK_B200_LIB", LIB_PATH))
        if not path.exists():
            raise RuntimeError(
                f"CUDA library {path} is missing: build it with "
                "`python -m polar_pack_b200.build` (there is no CPU fallback)")
        lib = ctypes.CDLL(str(path))
        for name, (args, res) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _lib = lib
    return _lib


class PolarPackError(RuntimeError):
    """A C-ABI call returned an error status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[polar_pack_b200 error {code}] {msg}")
        self.code = code


def check(rc: int) -> None:
    if rc != PP_OK:
        msg = load().pp_last_error().decode(errors="replace")
        if rc == PP_ERR_INVALID:
            raise ValueError(msg)
        raise PolarPackError(rc, msg)


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))


def ptr(t) -> int | None:
    if t is None:
        return None
    return t.data_ptr()


def ptrs(ts, n) -> ctypes.Array:
    arr = (_c_void_p * n)()
    for i, t in enumerate(ts):
        arr[i] = t.data_ptr()
    return arr


def floats4(vals) -> ctypes.Array:
    return _F4(*[float(v) for v in vals])


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors) -> torch.device:
    """All tensors on one CUDA device; the path has no CPU implementation."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("polar_pack_b200 kernels run on CUDA tensors only (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def set_launch_overlap(enable: bool) -> bool:
    """Programmatic dependent launch for the quad GEMV kernels and the
    decoder-step ops (process-wide).

    While on, the codes, tables and plug arrays of a call must not be
    written by the kernel launched immediately before it on the same
    stream; nor the norm weights of pp_rmsnorm_rows, nor the position and
    the cache rows before it of pp_decode_attention, by any kernel still
    running before them (a step sets its position before its first launch).
    Returns the previous setting.
    """
    return bool(load().pp_set_launch_overlap(1 if enable else 0))


# -------------------------------------------------------- prepared tables --
_tables: dict = {}
_TABLES_MAX = 64


def prepare_tables(luts, device: torch.device) -> torch.Tensor:
    """The 128 KiB replicated-table image of seven FP16[256] tables
    (``pp_quad_prepare_tables``), on the current stream of ``device``."""
    nbytes = _size_t()
    check(load().pp_quad_tables_bytes(ctypes.byref(nbytes)))
    t = torch.empty(nbytes.value, dtype=torch.uint8, device=device)
    call("pp_quad_prepare_tables", ptrs(luts, 7), t.data_ptr(), stream_handle(device))
    return t


def cached_tables(luts, device: torch.device) -> torch.Tensor:
    """Prepared tables for ``luts``, cached by the tensors' storage address
    and version counter (an in-place change of a table misses the cache).
    Each entry keeps references to its seven tensors, so no other tensor can
    take over one of those addresses while the entry exists."""
    key = (device.index,) + tuple((t.data_ptr(), t._version) for t in luts)
    hit = _tables.get(key)
    if hit is None:
        if len(_tables) >= _TABLES_MAX:
            _tables.pop(next(iter(_tables)))
        hit = (list(luts), prepare_tables(luts, device))
        _tables[key] = hit
    return hit[1]


# ------------------------------------------------------------- workspace --
_ws: dict = {}


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Zero-filled scratch for split-K reductions, one per (device, stream).

    Kernels leave their counters at zero, so the buffer is reused as is by
    later calls on the same stream; it only grows.
    """
    stream = torch.cuda.current_stream(device)
    key = (device.index, stream.cuda_stream)
    buf = _ws.get(key)
    if buf is None or buf.numel() < nbytes:
        size = max(nbytes, 1 << 20)
        buf = torch.zeros(size, dtype=torch.uint8, device=device)
        _ws[key] = buf
    return buf
