"""Decoder-step ops between the packed Linears (``csrc/decode_ops.cu``) against
torch restatements of the Qwen2 modules' FP16 steps.

* RMSNorm ``fp16(w * fp16(x * rsqrt(mean(x^2) + eps)))`` with FP32
  statistics: within one FP16 step of the restatement (the FP32 sum runs in
  another order); the interleaved copy equals the rows exactly.
* SwiGLU ``fp16(fp16(silu(g)) * u)`` with SiLU in FP32: within one FP16 step
  (``expf`` against torch's exp); even widths take the paired path, odd ones
  the single-element path; the interleaved copy equals the rows exactly.
* Embedding rows gathered exactly; a token outside the vocabulary gives a
  zero row and status 4.
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ulp_close(a: torch.Tensor, b: torch.Tensor, steps: int = 1) -> bool:
    """|a - b| within `steps` FP16 steps of max(|a|, |b|) (normal range)."""
    a, b = a.float(), b.float()
    m = torch.maximum(a.abs(), b.abs()).clamp_min(2.0 ** -14)
    step = torch.exp2(torch.floor(torch.log2(m)) - 10)
    return bool(((a - b).abs() <= steps * step).all())


@pytest.mark.parametrize("H", [2048, 3584, 4200])
def test_rmsnorm_rows(cuda, H):
    from polar_pack_b200 import _lib
    g = torch.Generator(device=cuda).manual_seed(H)
    x = (torch.randn(4, H, generator=g, device=cuda) * 3).half()
    w = (torch.randn(4, H, generator=g, device=cuda) * 0.1 + 1).half()
    y = torch.empty(4, H, dtype=torch.float16, device=cuda)
    y_il = torch.empty(4 * H, dtype=torch.float16, device=cuda)
    eps = 1e-6
    _lib.call("pp_rmsnorm_rows", x.data_ptr(), H, _lib.ptrs(list(w), 4), H, eps, y.data_ptr(), H, y_il.data_ptr(),
              None, 0, None, None, _lib.stream_handle(cuda))
    torch.cuda.synchronize(cuda)
    xf = x.float()
    r = torch.rsqrt((xf * xf).mean(dim=1, keepdim=True) + eps)
    ref = (w.float() * (xf * r).half().float()).half()
    assert _ulp_close(y, ref)
    assert torch.equal(y_il.view(H, 4).t(), y)


@pytest.mark.parametrize("I", [11008, 18944, 1001])
def test_swiglu_rows(cuda, I):
    from polar_pack_b200 import _lib
    g = torch.Generator(device=cuda).manual_seed(I)
    gu = (torch.randn(4, 2 * I, generator=g, device=cuda) * 2).half()
    y = torch.empty(4, I, dtype=torch.float16, device=cuda)
    y_il = torch.empty(4 * I + 8, dtype=torch.float16, device=cuda)
    _lib.call("pp_swiglu_rows", gu.data_ptr(), 2 * I, I, y.data_ptr(), I, y_il.data_ptr(), None, 0, None, None,
              _lib.stream_handle(cuda))
    torch.cuda.synchronize(cuda)
    gf = gu[:, :I].float()
    ref = ((gf / (1 + torch.exp(-gf))).half().float() * gu[:, I:].float()).half()
    assert _ulp_close(y, ref)
    assert torch.equal(y_il[:4 * I].view(I, 4).t(), y)


def test_embed_rows(cuda):
    from polar_pack_b200 import _lib
    V, H = 1000, 512
    g = torch.Generator(device=cuda).manual_seed(5)
    tables = [(torch.randn(V, H, generator=g, device=cuda) * 0.02).half() for _ in range(4)]
    tokens = torch.tensor([3, 999, 0, 1000], dtype=torch.int32, device=cuda)   # the last is out of range
    h = torch.full((4, H), 7.0, dtype=torch.float16, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    _lib.call("pp_embed_rows", tokens.data_ptr(), _lib.ptrs(tables, 4), V, H, h.data_ptr(), H, status.data_ptr(),
              _lib.stream_handle(cuda))
    torch.cuda.synchronize(cuda)
    for m, t in enumerate([3, 999, 0]):
        assert torch.equal(h[m], tables[m][t])
    assert torch.equal(h[3], torch.zeros(H, dtype=torch.float16, device=cuda))
    assert int(status.item()) == 4
