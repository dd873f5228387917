"""Decode attention with RoPE and the KV-cache append (``pp_decode_attention``)
against a float32 restatement of the Qwen2 attention step.

The queries and the token's key are rotated with the FP16 steps of the HF
modules (q' = fp16(fp16(q cos) + fp16(rotate_half(q) sin))); the appended cache
row must equal that rotation bit for bit, and the attention output must match
``softmax(q k^T / sqrt(d)) v`` computed in float32 from the same FP16 inputs
within 2e-3 of max|v| (the kernel rounds the softmax weights to FP16 before
the value product, 2^-11 relative, and rounds the output to FP16).

Cases cover grouped-query shapes of the Qwen2 family (2, 7, 8 query heads per
kv head) and the 16-head tile pair, positions on and around the 32-position
tile edges, split counts whose warps own one or several tiles, and a run of
consecutive positions that reads rows appended by earlier launches.
"""
from __future__ import annotations

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 2e-3
HD = 128


def _tables(max_pos, device, theta=1_000_000.0):
    inv = 1.0 / (theta ** (torch.arange(0, HD, 2, dtype=torch.int64).float() / HD))
    f = torch.arange(max_pos, dtype=torch.float32)[:, None] * inv[None, :]
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().half().to(device), emb.sin().half().to(device)


def _rope(x, c, s):
    """FP16 rotation of x [..., HD] with cos / sin rows c, s (FP16)."""
    rot = torch.cat([-x[..., HD // 2:], x[..., :HD // 2]], dim=-1)
    return (x * c) + (rot * s)          # FP16 products and sum, each rounded (torch half arithmetic)


class _Attn:
    def __init__(self, nq, nkv, max_pos, splits, device):
        from polar_pack_b200 import _lib
        self.lib, self._lib = _lib.load(), _lib
        self.nq, self.nkv, self.max_pos, self.splits, self.dev = nq, nkv, max_pos, splits, device
        self.cos, self.sin = _tables(max_pos, device)
        g = torch.Generator(device=device)
        g.manual_seed(nq * 1000 + nkv * 10 + splits)
        self.g = g
        self.kc = torch.zeros(4, max_pos, nkv, HD, dtype=torch.float16, device=device)
        self.vc = torch.zeros_like(self.kc)
        nb = _lib._size_t()
        _lib.check(self.lib.pp_decode_attention_workspace_bytes(nq, nkv, splits, ctypes.byref(nb)))
        self.ws = torch.zeros(nb.value, dtype=torch.uint8, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.pos = torch.zeros(1, dtype=torch.int32, device=device)
        self.out = torch.zeros(4, nq * HD, dtype=torch.float16, device=device)
        self.out_il = torch.zeros(4 * nq * HD, dtype=torch.float16, device=device)
        P4 = _lib._PTR4
        self._kc = P4(*[self.kc[k].data_ptr() for k in range(4)])
        self._vc = P4(*[self.vc[k].data_ptr() for k in range(4)])

    def fill(self, upto):
        """Random rotated keys and values at positions [0, upto)."""
        r = lambda: (torch.randn(4, upto, self.nkv, HD, generator=self.g, device=self.dev) * 0.5).half()
        self.kc[:, :upto] = r()
        self.vc[:, :upto] = r()

    def step(self, pos):
        qkv = (torch.randn(4, (self.nq + 2 * self.nkv) * HD, generator=self.g, device=self.dev) * 0.5).half()
        self.pos.fill_(pos)
        self._lib.check(self.lib.pp_decode_attention(
            qkv.data_ptr(), qkv.stride(0), self.nq, self.nkv, HD, self.cos.data_ptr(), self.sin.data_ptr(),
            self._kc, self._vc, self.max_pos, self.pos.data_ptr(), 1.0 / math.sqrt(HD), self.out.data_ptr(),
            self.out.stride(0), self.out_il.data_ptr(), self.splits, self.ws.data_ptr(), self.ws.numel(),
            self.status.data_ptr(),
            None, 0, None, None, self._lib.stream_handle(self.dev)))
        torch.cuda.synchronize(self.dev)
        return qkv

    def check(self, qkv, pos):
        nq, nkv, grp = self.nq, self.nkv, self.nq // self.nkv
        c, s = self.cos[pos], self.sin[pos]
        q = _rope(qkv[:, :nq * HD].view(4, nq, HD), c, s)
        k_new = _rope(qkv[:, nq * HD:(nq + nkv) * HD].view(4, nkv, HD), c, s)
        v_new = qkv[:, (nq + nkv) * HD:].view(4, nkv, HD)
        assert torch.equal(self.kc[:, pos], k_new), "appended key row differs from the FP16 rotation"
        assert torch.equal(self.vc[:, pos], v_new), "appended value row differs"
        K = self.kc[:, :pos + 1].float()                    # [4, t, nkv, HD]
        V = self.vc[:, :pos + 1].float()
        kv_of = torch.arange(nq, device=self.dev) // grp
        sc = torch.einsum("mhd,mthd->mht", q.float(), K[:, :, kv_of]) / math.sqrt(HD)
        ref = torch.einsum("mht,mthd->mhd", torch.softmax(sc, -1), V[:, :, kv_of])
        got = self.out.view(4, nq, HD).float()
        err = float((got - ref).abs().max() / V.abs().max())
        assert err <= TOL, (pos, err)
        assert torch.equal(self.out_il.view(-1, 4).t(), self.out)      # interleaved copy
        assert int(self.status.item()) == 0


@pytest.mark.parametrize("nq,nkv", [(4, 2), (16, 2), (28, 4), (32, 2)])
@pytest.mark.parametrize("splits", [1, 3, 8])
def test_attention_positions(cuda, nq, nkv, splits):
    a = _Attn(nq, nkv, max_pos=1100, splits=splits, device=cuda)
    a.fill(1100)
    for pos in (0, 1, 30, 31, 32, 33, 63, 64, 255, 256, 257, 1000, 1099):
        a.check(a.step(pos), pos)


def test_attention_consecutive_positions(cuda):
    """Rows appended by earlier launches are the ones later launches read."""
    a = _Attn(16, 2, max_pos=96, splits=2, device=cuda)
    for pos in range(70):
        a.check(a.step(pos), pos)


def test_attention_position_out_of_range_sets_status(cuda):
    a = _Attn(4, 2, max_pos=64, splits=2, device=cuda)
    a.step(64)
    assert int(a.status.item()) == 5


def test_attention_rejects_unsupported_groups(cuda):
    from polar_pack_b200 import _lib
    a = _Attn(4, 2, max_pos=64, splits=2, device=cuda)
    with pytest.raises(ValueError):
        _lib.check(a.lib.pp_decode_attention(
            a.out.data_ptr(), 0, 34, 2, HD, a.cos.data_ptr(), a.sin.data_ptr(), a._kc, a._vc, 64,
            a.pos.data_ptr(), 1.0, a.out.data_ptr(), a.out.stride(0), None, 2, a.ws.data_ptr(), a.ws.numel(),
            a.status.data_ptr(), None, 0, None, None, _lib.stream_handle(a.dev)))
