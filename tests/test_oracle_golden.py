"""Pin the CPU oracle (and the host-side packers) to the reference's own outputs.

The fixtures were produced by running the reference (tests/golden/make_golden.py):
its packers, its numpy unpackers, and its Triton kernels under the Triton CPU
interpreter.  CPU only.
"""
from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from conftest import bits
from oracle import dual as od
from oracle import formats as of
from oracle import quad as oq

QUAD_TAGS = ("a", "b", "c")
DUAL_TAGS = ("a", "b")


def _quad_case(g, tag):
    codes = g[f"{tag}_codes"]
    luts = [g[f"{tag}_lut{i}"] for i in range(7)]
    return codes, luts, g[f"{tag}_scales"]


@pytest.mark.parametrize("tag", QUAD_TAGS)
def test_quad_decode_matches_reference_kernel(quad_golden, tag):
    codes, luts, _ = _quad_case(quad_golden, tag)
    dec = oq.decode_quad_fp16(codes, luts)
    for k in range(4):
        # the reference decode was read back through a @ I, which turns -0 into +0
        np.testing.assert_array_equal(dec[k].astype(np.float32), quad_golden[f"{tag}_dec{k}"].astype(np.float32))


@pytest.mark.parametrize("tag", QUAD_TAGS)
@pytest.mark.parametrize("M", [1, 5])
def test_quad_gemm_matches_reference_kernel(quad_golden, tag, M):
    codes, luts, scales = _quad_case(quad_golden, tag)
    out = oq.quad_gemm(quad_golden[f"{tag}_a{M}"], codes, luts, scales)
    for k in range(4):
        assert oq.rel_err(quad_golden[f"{tag}_out{M}_{k}"], out[k]) <= 1e-3


@pytest.mark.parametrize("tag", QUAD_TAGS)
def test_quad_packers_match_reference(quad_golden, tag):
    codes, luts, scales = _quad_case(quad_golden, tag)
    ws = [quad_golden[f"{tag}_w{k}"] for k in range(4)]
    # numpy restatement
    c2, l2, s2 = oq.pack_quad_layer(*ws)
    assert np.mean(c2 != codes) <= 1e-3
    for a, b in zip(l2, luts):
        np.testing.assert_array_equal(bits(a), bits(b))
    np.testing.assert_allclose(s2, scales, rtol=1e-6)
    # product host packer (torch, CPU): same ops as the reference -> identical
    from polar_pack_b200.quad_kernels import pack_quad_layer
    c3, l3, s3 = pack_quad_layer(*[torch.from_numpy(w) for w in ws])
    assert c3.dtype == torch.uint32
    np.testing.assert_array_equal(c3.numpy(), codes)
    for a, b in zip(l3, luts):
        np.testing.assert_array_equal(bits(a.numpy()), bits(b))
    assert s3 == pytest.approx(list(scales), rel=0, abs=0)


@pytest.mark.parametrize("tag", DUAL_TAGS)
def test_dual_decode_and_gemm_match_reference_kernel(dual_golden, tag):
    g = dual_golden
    args = [g[f"{tag}_bmax"], g[f"{tag}_amp_lut"], g[f"{tag}_cos_lut"], g[f"{tag}_sin_lut"]]
    dec = od.decode_dual_fp16(g[f"{tag}_packed"], *args)
    for j in range(2):
        np.testing.assert_array_equal(dec[j].astype(np.float32), g[f"{tag}_dec{j}"].astype(np.float32))
    for M in (1, 4):
        out = od.dual_gemm(g[f"{tag}_a{M}"], g[f"{tag}_packed"], *args)
        for j in range(2):
            assert oq.rel_err(g[f"{tag}_out{M}_{j}"], out[j]) <= 1e-3


@pytest.mark.parametrize("tag", DUAL_TAGS)
def test_dual_packers_match_reference(dual_golden, tag):
    g = dual_golden
    w1, w2 = g[f"{tag}_w0"].astype(np.float32), g[f"{tag}_w1"].astype(np.float32)
    ref = [g[f"{tag}_packed"], g[f"{tag}_bmax"], g[f"{tag}_amp_lut"], g[f"{tag}_cos_lut"], g[f"{tag}_sin_lut"]]
    mine = od.quantize_polar_bitpacked(w1, w2)
    np.testing.assert_array_equal(mine[0], ref[0])
    for a, b in zip(mine[1:], ref[1:]):
        np.testing.assert_array_equal(bits(a), bits(b))
    from polar_pack_b200.polar_kernels import quantize_polar_bitpacked
    prod = quantize_polar_bitpacked(torch.from_numpy(w1), torch.from_numpy(w2))
    np.testing.assert_array_equal(prod[0].numpy(), ref[0])
    for a, b in zip(prod[1:], ref[1:]):
        np.testing.assert_array_equal(bits(a.numpy()), bits(b))


def test_pack_amp_phase_all_codes(dual_golden):
    aq = np.repeat(np.arange(64), 1024)
    pq = np.tile(np.arange(1024), 64)
    np.testing.assert_array_equal(od.pack_amp_phase(aq, pq), dual_golden["amp_phase_all"])
    from polar_pack_b200.polar_kernels import pack_amp_phase
    np.testing.assert_array_equal(pack_amp_phase(torch.from_numpy(aq), torch.from_numpy(pq)).numpy(),
                                  dual_golden["amp_phase_all"])


def test_dualpack_stream_roundtrip(dualpack_golden):
    g = dualpack_golden
    buf = g["stream"].tobytes()
    out = of.unpack_dual_bytes(buf)
    np.testing.assert_array_equal(out[0], g["restored1"])
    np.testing.assert_array_equal(out[1], g["restored2"])
    amp_bits, num_phases, mu, gs, chunk = (int(x) for x in g["config"])
    again = of.pack_dual_bytes(g["w1"], g["w2"], amp_bits, num_phases, mu, gs, chunk, float(g["plug_cap"]))
    assert again == buf


def test_quadpack_header_and_windows(quadpack_golden):
    g = quadpack_golden
    hdr = of.parse_quad_header(g["header"].tobytes())
    seed, n, *extra = (int(x) for x in g["seed_models"])
    assert hdr["n"] == n and hdr["tails"] == extra and hdr["n_models"] == 4
    assert of.QUAD_HEADER_SIZE == 82
    off = of.quad_offsets(hdr)
    assert off["tails"] + 2 * sum(extra) == int(g["size"])
    # decode each window with the plug entries inside it
    for tag in ("w0", "w1"):
        lo, hi = (int(x) for x in g[f"{tag}_range"])
        window = g[f"{tag}_codes"]
        pidx = g[f"{tag}_pidx"].astype(np.int64) - lo
        pval = g[f"{tag}_pval"]
        # build a tiny standalone stream holding just this window
        import struct
        h = list(struct.unpack(of.QUAD_HEADER_FMT, g["header"].tobytes()))
        h[3] = hi - lo
        h[9] = len(pidx)
        h[15:19] = [0, 0, 0, 0]
        buf = struct.pack(of.QUAD_HEADER_FMT, *h) + window.tobytes() + \
            pidx.astype(np.uint32).tobytes() + pval.tobytes()
        rest = of.unpack_quad_bytes(buf)
        for k in range(4):
            np.testing.assert_array_equal(rest[k], g[f"{tag}_restored{k}"])
    tails = np.frombuffer(g["tails_raw"].tobytes(), np.float16)
    o = 0
    for k in range(4):
        t = extra[k]
        np.testing.assert_array_equal(tails[o:o + t].astype(np.float32), g[f"tail_restored{k}"])
        o += t


@pytest.mark.slow
def test_quadpack_writer_reproduces_reference_stream(quadpack_golden):
    """The oracle's writer produces the reference's exact bytes (SHA-256)."""
    from make_golden import correlated_models
    g = quadpack_golden
    seed, n, *extra = (int(x) for x in g["seed_models"])
    flat = correlated_models(np.random.default_rng(seed), 4, (n + max(extra),))
    models = [flat[k][: n + extra[k]].astype(np.float32) for k in range(4)]
    buf = of.pack_quad_bytes(models)
    assert len(buf) == int(g["size"])
    assert hashlib.sha256(buf).hexdigest() == str(g["sha256"])
    rest = of.unpack_quad_bytes(buf)
    for tag in ("w0", "w1"):
        lo, hi = (int(x) for x in g[f"{tag}_range"])
        for k in range(4):
            np.testing.assert_array_equal(rest[k][lo:hi], g[f"{tag}_restored{k}"])
