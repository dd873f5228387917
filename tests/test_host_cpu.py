"""Host-side logic that needs no GPU: the C-ABI library, argument checks, readers."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from oracle import formats as of

ROOT = Path(__file__).resolve().parent.parent


def header_symbols() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        names |= set(re.findall(r"PP_API\s+[\w\s\*]*?\b(pp_\w+)\s*\(", h.read_text()))
    return names


def test_library_loads_and_exports_every_declared_symbol():
    from polar_pack_b200 import _lib
    lib = _lib.load()
    declared = header_symbols()
    assert len(declared) >= 13
    for name in declared:
        assert hasattr(lib, name), name
    assert declared == set(_lib.exported_symbols())
    assert lib.pp_version() == 1


def test_invalid_arguments_rejected_on_host():
    from polar_pack_b200 import _lib
    lib = _lib.load()
    PTR7 = ctypes.c_void_p * 7
    PTR4 = ctypes.c_void_p * 4
    F4 = ctypes.c_float * 4
    rc = lib.pp_quad_gemm(None, 0, 0, None, 0, 0, PTR7(*([1] * 7)), F4(1, 1, 1, 1), PTR4(*([1] * 4)),
                          0, 0, -1, 4, 4, None, 0, None)
    assert rc == _lib.PP_ERR_INVALID
    assert b"negative" in lib.pp_last_error()
    rc = lib.pp_quad_gemm(None, 0, 0, None, 0, 0, PTR7(*([1] * 6 + [0])), F4(1, 1, 1, 1),
                          PTR4(*([1] * 4)), 0, 0, 1, 4, 4, None, 0, None)
    assert rc == _lib.PP_ERR_INVALID and b"luts[6]" in lib.pp_last_error()
    rc = lib.pp_dual_gemm(None, 0, 0, None, 0, 0, None, 0, None, None, None, None, None, 0, 0,
                          1, 1, 1, None, 0, None)
    assert rc == _lib.PP_ERR_INVALID
    with pytest.raises(ValueError):
        _lib.check(rc)


def test_workspace_size_queries_without_gpu():
    from polar_pack_b200 import _lib
    lib = _lib.load()
    n = ctypes.c_size_t()
    assert lib.pp_quad_gemm_workspace_bytes(1, 2048, 2048, 2048, 1, ctypes.byref(n)) == 0
    assert n.value > 0 and n.value % 4 == 0
    assert lib.pp_quad_linear_workspace_bytes(0, 2048, 2048, ctypes.byref(n)) == 0 and n.value == 0
    assert lib.pp_dual_gemm_workspace_bytes(16, 256, 4096, 256, 1, ctypes.byref(n)) == 0 and n.value > 0


def test_quadpack_reader(quadpack_golden):
    from polar_pack_b200.quadpack import HEADER_SIZE, QuadHeader
    g = quadpack_golden
    h = QuadHeader.parse(g["header"].tobytes())
    ref = of.parse_quad_header(g["header"].tobytes())
    assert HEADER_SIZE == of.QUAD_HEADER_SIZE == 82
    assert (h.n, h.plug_n, h.tails, h.r_max) == (ref["n"], ref["plug_n"], ref["tails"], ref["r_max"])
    assert h.offsets()["end"] == int(g["size"])
    with pytest.raises(ValueError):
        QuadHeader.parse(b"XXXX" + g["header"].tobytes()[4:])
    with pytest.raises(ValueError):
        QuadHeader.parse(g["header"].tobytes()[:40])


def test_quadpack_file_views_small_stream():
    from polar_pack_b200.quadpack import QuadPackFile
    rng = np.random.default_rng(1)
    models = [rng.normal(0, 0.02, 5000 + e).astype(np.float32) for e in (0, 7, 0, 3)]
    buf = of.pack_quad_bytes(models, plug_cap=0.05, threshold_windows=4, window=1000)
    f = QuadPackFile(buf)
    hdr, codes, pidx, pval, tails = of.quad_sections(buf)
    np.testing.assert_array_equal(f.codes, codes)
    np.testing.assert_array_equal(f.plug_vals, pval)
    assert [t.size for t in f.tails] == [0, 7, 0, 3]
    lo, hi = f.plug_range(100, 900)
    assert np.all((f.plug_pos[lo:hi] >= 100) & (f.plug_pos[lo:hi] < 900))
    with pytest.raises(ValueError):
        QuadPackFile(buf[:-1])


def test_wrapped_plug_positions():
    from polar_pack_b200.quadpack import unwrap_u32_positions
    true = np.array([5, 2 ** 32 - 3, 2 ** 32 + 7, 2 ** 33 + 1], dtype=np.int64)
    stored = (true & 0xFFFFFFFF).astype(np.uint32)
    np.testing.assert_array_equal(unwrap_u32_positions(stored), true)


def test_layer_offsets_follow_map_order():
    from polar_pack_b200.quadpack import layer_offsets
    m = [{"name": "a", "shape": [4, 8], "numel": 32}, {"name": "b", "shape": [2, 8], "numel": 16},
         {"name": "c", "shape": [8, 2], "numel": 16}]
    assert layer_offsets(m) == [("a", 0, (4, 8)), ("b", 32, (2, 8)), ("c", 48, (8, 2))]


def test_product_never_imports_oracle():
    pkg = ROOT / "polar_pack_b200"
    for p in pkg.rglob("*.py"):
        src = p.read_text()
        assert "import oracle" not in src and "from oracle" not in src, p


def test_tail_split_rows():
    """Row split of a Linear at n_min (quaternion_packer.py:55-57, 118-126)."""
    from polar_pack_b200.quadpack import tail_split
    n, tails = 1000, [0, 40, 0, 17]
    s = tail_split(980, 7, 8, n, tails)             # rows 0,1 coded, row 2 cut, rows 3.. tail
    assert (s.coded, s.straddle, s.first_tail, s.tail_start) == (2, True, 3, 4)
    assert s.present == (False, True, False, False)
    s = tail_split(988, 7, 4, n, tails)             # rows end exactly at n_min
    assert (s.coded, s.straddle, s.first_tail, s.tail_start) == (3, False, 3, 0)
    assert s.present == (False, True, False, True)
    s = tail_split(1008, 4, 8, n, tails)            # wholly in the tails
    assert (s.coded, s.straddle, s.first_tail, s.tail_start) == (0, False, 0, 8)
    s = tail_split(0, 10, 8, n, tails)              # wholly coded
    assert (s.coded, s.straddle) == (10, False) and all(s.present)


def test_dualpack_reader(dualpack_golden):
    """Product reader of .dualpack v2 against the oracle's section parser
    (polar_bitpack.py:26-29, 194-215)."""
    from polar_pack_b200.dualpack import DualPackFile, dual_tables
    buf = dualpack_golden["stream"].tobytes()
    f = DualPackFile(buf)
    hdr, codes, scales, pidx, pval = of.dual_sections(buf)
    h = f.header
    assert (h.n_pairs, h.n1, h.n2, h.amp_bits, h.phase_bits, h.group_size, h.chunk_size, h.plug_n) == \
        (hdr["n_pairs"], hdr["n1"], hdr["n2"], hdr["amp_bits"], hdr["phase_bits"], hdr["group_size"],
         hdr["chunk_size"], hdr["plug_n"])
    be = (f.codes[0::2].astype(np.uint32) << 8) | f.codes[1::2]
    np.testing.assert_array_equal(be, codes)
    np.testing.assert_array_equal(f.scales.view(np.uint16), scales.view(np.uint16))
    np.testing.assert_array_equal(f.plug_idx, pidx)
    amp, c, s = dual_tables(h)
    assert amp[0] == 0.0 and amp.size == 2 ** h.amp_bits and c.size == 2 ** h.phase_bits
    with pytest.raises(ValueError):
        DualPackFile(buf[:70])
