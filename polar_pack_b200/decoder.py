"""Packed Linears in models: the loader, and a 4-model decoder step.

Two ways to serve the Linears of a ``.quadpack`` from HBM without unpacking:

* :func:`replace_model_weights_packed` is the counterpart of the reference's
  integration point ``replace_model_weights`` (polar_packer.py:285-316): it
  walks the layer map of ``collect_weights`` (polar_main.py:25-51) over a
  model's ``named_modules`` and installs a :class:`PackedQuadLinear` where the
  reference overwrites ``nn.Linear.weight`` with unpacked FP16 weights.  Each
  forward streams the packed codes (one pass yields all four models; the
  module returns its model's output) and keeps the module's own bias.
* :class:`QuadDecoder` runs one decoder step of the four packed models at
  once -- one token per model, each model with its own hidden state -- for a
  Qwen2-style architecture (the reference's models: polar_inference.py
  generates through Hugging Face Qwen2 modules).  Every packed Linear is one
  launch over its codes that multiplies model k's weights with model k's row
  (``PP_QUAD_PER_MODEL_X``), with the q/k/v bias and the residual add in its
  epilogue; RMSNorm, decode attention (with the rotary embedding and the
  KV-cache append fused in) and SwiGLU are this library's kernels
  (``decode_ops.cu``).  The step has fixed
  buffers and a device-side position, so it can be captured once as a CUDA
  graph and replayed for every token.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch
import torch.nn as nn

from . import _lib
from .quadpack import QuadLinearGroup, QuadTailedLinear, layer_offsets, quad_linear


# --------------------------------------------------------------- loader ----
class PackedQuadLinear(nn.Module):
    """An ``nn.Linear`` whose weight is model ``model_index`` of a packed
    Linear (``QuadPackDevice.linear``): ``y = x W_k^T + b``.  The forward is
    one fused launch over the codes (``quad_linear``), or the tail path for a
    Linear past ``n_min``."""

    def __init__(self, layer, model_index: int, bias: torch.Tensor | None = None):
        super().__init__()
        self.layer = layer
        self.model_index = model_index
        self.in_features, self.out_features = layer.K, layer.N
        self.bias = nn.Parameter(bias.detach().to(torch.float16), requires_grad=False) if bias is not None else None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).to(torch.float16)
        if isinstance(self.layer, QuadTailedLinear):
            y = self.layer(x2)[self.model_index]
            if y is None:
                raise ValueError(f"model {self.model_index} has no weights for this Linear")
        else:
            y = quad_linear(x2, self.layer)[self.model_index]
        if self.bias is not None:
            y = y + self.bias
        return y.reshape(*shape[:-1], self.out_features)


def replace_model_weights_packed(model: nn.Module, pack, layer_map: list[dict], model_index: int) -> int:
    """Install packed Linears of model ``model_index`` into ``model``.

    Follows replace_model_weights (polar_packer.py:285-316): the flat offset
    of each layer-map entry is the running sum of ``numel``; an entry whose
    module is not an ``nn.Linear`` or whose weight size differs is skipped
    (its offset still advances).  The module is replaced in its parent by a
    :class:`PackedQuadLinear` that keeps the original bias.  Returns the number
    of modules replaced.
    """
    replaced = 0
    for (name, off, shape), info in zip(layer_offsets(layer_map), layer_map):
        parent, module = None, model
        parts = name.split(".")
        for part in parts:
            parent = module
            module = module[int(part)] if part.isdigit() else getattr(module, part)
        if not isinstance(module, nn.Linear) or module.weight.numel() != int(info["numel"]):
            continue
        N, K = shape
        packed = PackedQuadLinear(pack.linear(off, N, K), model_index, module.bias)
        if parts[-1].isdigit():
            parent[int(parts[-1])] = packed
        else:
            setattr(parent, parts[-1], packed)
        replaced += 1
    return replaced


# -------------------------------------------------------------- decoder ----
@dataclass
class DecoderConfig:
    layers: int
    hidden: int
    inter: int
    q_heads: int
    kv_heads: int
    vocab: int
    head_dim: int = 128
    rms_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    max_pos: int = 2048
    qkv_bias: bool = True

    @property
    def q_dim(self) -> int:
        return self.q_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim


def qwen2_layer_map(cfg: DecoderConfig) -> list[dict]:
    """The ``collect_weights`` layer map (polar_main.py:25-51: every
    ``nn.Linear`` in ``named_modules`` order) of a Qwen2 causal LM."""
    h, i = cfg.hidden, cfg.inter
    ents = []
    for l in range(cfg.layers):
        p = f"model.layers.{l}."
        for name, shape in ((p + "self_attn.q_proj", (cfg.q_dim, h)), (p + "self_attn.k_proj", (cfg.kv_dim, h)),
                            (p + "self_attn.v_proj", (cfg.kv_dim, h)), (p + "self_attn.o_proj", (h, cfg.q_dim)),
                            (p + "mlp.gate_proj", (i, h)), (p + "mlp.up_proj", (i, h)), (p + "mlp.down_proj", (h, i))):
            ents.append({"name": name, "shape": list(shape), "numel": shape[0] * shape[1]})
    ents.append({"name": "lm_head", "shape": [cfg.vocab, h], "numel": cfg.vocab * h})
    return ents


def rope_tables(cfg: DecoderConfig, device) -> tuple[torch.Tensor, torch.Tensor]:
    """FP16 cos / sin ``[max_pos][head_dim]`` of the Qwen2 rotary embedding:
    ``inv_freq = 1 / theta^(2j/d)`` in FP32, ``emb = cat(pos * inv_freq,
    pos * inv_freq)``, cos / sin in FP32 rounded to FP16."""
    d = cfg.head_dim
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2, dtype=torch.int64).float() / d))
    pos = torch.arange(cfg.max_pos, dtype=torch.float32)
    freqs = pos[:, None] * inv[None, :]
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().half().to(device), emb.sin().half().to(device)


@dataclass
class DecoderExtras:
    """The per-model weights that are not packed Linears (FP16, [4][...])."""
    embed: torch.Tensor        # [4][vocab][hidden]
    in_norm: torch.Tensor      # [layers][4][hidden]
    post_norm: torch.Tensor    # [layers][4][hidden]
    final_norm: torch.Tensor   # [4][hidden]
    qkv_bias: torch.Tensor | None  # [layers][4][q + 2 kv]

    @staticmethod
    def random(cfg: DecoderConfig, device, seed: int = 0) -> "DecoderExtras":
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        H, L = cfg.hidden, cfg.layers
        r = lambda *s, sd=1.0, mean=0.0: (torch.randn(*s, generator=g, device=device) * sd + mean).half()
        return DecoderExtras(embed=r(4, cfg.vocab, H, sd=0.02), in_norm=r(L, 4, H, sd=0.05, mean=1.0),
                             post_norm=r(L, 4, H, sd=0.05, mean=1.0), final_norm=r(4, H, sd=0.05, mean=1.0),
                             qkv_bias=r(L, 4, cfg.q_dim + 2 * cfg.kv_dim, sd=0.02) if cfg.qkv_bias else None)


def fused_rows(N: int, K: int, sms: int) -> list[tuple[int, int]]:
    """Row chunks [r0, r1) of a Linear small enough for one fused launch each
    (each of the 16 warps of an SM holds at most 63 work units of 8 rows x
    64 codes), as equal as multiples of 8 rows allow."""
    units_per_row8 = -(-K // 64)
    cap_rows = max(8, (sms * 16 * 63 * 9 // 10) // units_per_row8 * 8)
    n = -(-N // cap_rows)
    step = -(-(-(-N // n)) // 8) * 8
    return [(r0, min(N, r0 + step)) for r0 in range(0, N, step)]


def linear_chunks(pack, offset: int, N: int, K: int, sms: int, x, out, bias=None, resid=None, x_il=None):
    """One per-model-activation group launch per row chunk of the Linear at
    ``offset`` (``out`` / ``bias`` / ``resid``: [4][N] tensors, or None;
    ``x_il``: the activations interleaved, see ``linear_desc``)."""
    res = []
    for r0, r1 in fused_rows(N, K, sms):
        cut = lambda t: [t[k:k + 1, r0:r1] for k in range(4)] if t is not None else None
        cutb = [bias[k][r0:r1] for k in range(4)] if bias is not None else None
        g = QuadLinearGroup([pack.linear(offset + r0 * K, r1 - r0, K)], [x], [cut(out)], per_model_x=True,
                            biases=[cutb], resids=[cut(resid)], x_ils=[x_il])
        if not g.single_launch:
            raise ValueError(f"rows [{r0}, {r1}) of the Linear at {offset} do not fit one fused launch")
        res.append(g)
    return res


class GatheredLinear:
    """This rank's row shard of a packed Linear with per-model activations,
    its outputs gathered into every rank's buffer (``peers`` buffer ``b``,
    viewed ``[4][N]``) by the GEMV itself, then one bounded wait.

    The shard runs in as many row chunks as the largest shard of any rank
    needs (one fused launch each), so that every rank makes the same number
    of launches into the buffer -- the wait compares launch counts.
    ``bias`` / ``resid``: four ``[N]`` vectors (the shard's rows are used)."""

    def __init__(self, pack, offset, N, K, sms, x, peers, b, world, rank, bias=None, resid=None, x_il=None):
        import ctypes as C

        from .parallel import row_shard, shard_width
        from .quadpack import linear_desc
        n0, n1 = row_shard(N, world, rank)
        nch = len(fused_rows(shard_width(N, world), K, sms))
        step = -(-(-(-(n1 - n0) // nch)) // 8) * 8
        self.peers, self.b, self.lib = peers, b, _lib.load()
        self.outs = (C.c_void_p * 8)(*peers.out_ptrs(b))
        self.flags = (C.c_void_p * 8)(*peers.flag_ptrs(b))
        self.calls, self._keep = [], []
        for c in range(nch):
            r0 = n0 + c * step
            r1 = min(n1, r0 + step)
            if r1 <= r0:
                raise ValueError("a rank's shard is too small for the common number of row chunks")
            lin = pack.linear(offset + r0 * K, r1 - r0, K)
            bb = [bias[k][r0:r1] for k in range(4)] if bias is not None else None
            rr = [resid[k:k + 1, r0:r1] for k in range(4)] if resid is not None else None
            d = (_lib.QuadLinearDesc * 1)(linear_desc(x, lin, None, True, bb, rr, x_il))
            if not self.lib.pp_quad_linear_group_single_launch(1, d):
                raise ValueError("a shard chunk does not fit one fused launch")
            nb = _lib._size_t()
            _lib.check(self.lib.pp_quad_linear_group_workspace_bytes(1, d, C.byref(nb)))
            ws = torch.zeros(max(nb.value, 256), dtype=torch.uint8, device=x.device)
            self.calls.append((d, (C.c_int64 * 1)(r0), ws))
            self._keep.append((lin, bb, rr))
        self.N = N

    def __call__(self, s) -> None:
        """The shard's launches; the reader of the buffer waits for every rank
        (``wait_args``), either inside its own kernel or with ``peers.wait``."""
        p = self.peers
        for d, row0, ws in self.calls:
            rc = self.lib.pp_quad_linear_group_gather(1, d, p.world, self.outs, self.N, row0, self.flags,
                                                      p.epoch_ptr(self.b), ws.data_ptr(), ws.numel(), s)
            if rc:
                _lib.check(rc)


class QuadDecoder:
    """One decoder step of the four models of a ``.quadpack`` on one GPU.

    ``pack`` is a :class:`~polar_pack_b200.quadpack.QuadPackDevice` whose
    stream holds the Linears of ``cfg`` in ``qwen2_layer_map`` order (q, k, v
    and gate, up are consecutive with one input, so each pair or triple is
    one launch).  ``step(tokens)`` takes one token id per model and returns
    ``logits`` ``[4][vocab]`` (FP16); the position advances by one per step.

    With ``world > 1`` (one process per GPU, ``torch.distributed`` set up) the
    packed Linears are row-sharded: each rank streams its rows of every
    Linear and stores its outputs into every rank's buffers over NVLink
    (:class:`GatheredLinear`); norms, attention and SwiGLU run on every rank
    over the gathered activations, so every rank holds the whole step's
    state and the logits.
    """

    def __init__(self, pack, cfg: DecoderConfig, extras: DecoderExtras, attn_splits: int | None = None, world: int = 1,
                 rank: int = 0):
        self.pack, self.cfg, self.ex = pack, cfg, extras
        dev = self.device = pack.device
        self.lib = _lib.load()
        H, I, V = cfg.hidden, cfg.inter, cfg.vocab
        qkv_n = cfg.q_dim + 2 * cfg.kv_dim
        f16 = dict(dtype=torch.float16, device=dev)
        self.tokens = torch.zeros(4, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.world, self.rank = world, rank
        self.peers = None
        if world > 1:
            # the outputs of the packed Linears live in buffers every rank writes:
            # 0 qkv, 1 the residual stream h, 2 gate_up, 3 logits
            from .parallel import PeerBuffers
            self.peers = PeerBuffers(4 * max(qkv_n, H, 2 * I, V), nbuf=4, device=dev)
            view = lambda b, n: self.peers.view(b)[:4 * n].view(4, n)
            self.qkv, self.h, self.gu, self.logits = view(0, qkv_n), view(1, H), view(2, 2 * I), view(3, V)
        else:
            self.h = torch.zeros(4, H, **f16)
            self.qkv = torch.zeros(4, qkv_n, **f16)
            self.gu = torch.zeros(4, 2 * I, **f16)
            self.logits = torch.zeros(4, V, **f16)
        self.xn = torch.zeros(4, H, **f16)
        self.attn = torch.zeros(4, cfg.q_dim, **f16)
        self.act = torch.zeros(4, I, **f16)
        # the inputs of the large Linears (gate_up, down, lm_head) also
        # interleaved ([i][model]): their fused plug correction reads a
        # column's four activations with one load (x_il); the small q/k/v and
        # o Linears gain less than the extra stores cost
        self.xn_il = torch.zeros(4 * H, **f16)
        self.act_il = torch.zeros(4 * I, **f16)
        self.kc = [torch.zeros(4, cfg.max_pos, cfg.kv_heads, cfg.head_dim, **f16) for _ in range(cfg.layers)]
        self.vc = [torch.zeros(4, cfg.max_pos, cfg.kv_heads, cfg.head_dim, **f16) for _ in range(cfg.layers)]
        self.cos, self.sin = rope_tables(cfg, dev)
        # attention: position ranges per (model, kv head); by default one per
        # 256 positions of the cache (a CTA's eight 32-position warp tiles at
        # full length), at most as many as keep the launch's splits x kv heads
        # x 4 CTAs (one per SM: each holds ~147 KB of shared memory) in one wave
        sms = self.lib.pp_device_sm_count(dev.index if dev.index is not None else 0)
        wave = max(1, sms // (4 * cfg.kv_heads))
        self.splits = attn_splits if attn_splits else max(1, min(64, wave, -(-cfg.max_pos // 256)))
        nb = _lib._size_t()
        _lib.check(self.lib.pp_decode_attention_workspace_bytes(cfg.q_heads, cfg.kv_heads, self.splits,
                                                                ctypes.byref(nb)))
        self.attn_ws = torch.zeros(nb.value, dtype=torch.uint8, device=dev)
        offs = {n: (o, s) for n, o, s in layer_offsets(qwen2_layer_map(cfg))}
        self.groups = []   # per layer: launches (row chunks) of qkv, o, gate_up, down
        for l in range(cfg.layers):
            p = f"model.layers.{l}."
            oq, _ = offs[p + "self_attn.q_proj"]
            oo, _ = offs[p + "self_attn.o_proj"]
            og, _ = offs[p + "mlp.gate_proj"]
            od, _ = offs[p + "mlp.down_proj"]
            bias = [extras.qkv_bias[l, k] for k in range(4)] if extras.qkv_bias is not None else None
            if world > 1:
                pr = self.peers
                self.groups.append((
                    [GatheredLinear(pack, oq, qkv_n, H, sms, self.xn, pr, 0, world, rank, bias=bias)],
                    [GatheredLinear(pack, oo, H, cfg.q_dim, sms, self.attn, pr, 1, world, rank, resid=self.h)],
                    [GatheredLinear(pack, og, 2 * I, H, sms, self.xn, pr, 2, world, rank, x_il=self.xn_il)],
                    [GatheredLinear(pack, od, H, I, sms, self.act, pr, 1, world, rank, resid=self.h,
                                    x_il=self.act_il)]))
            else:
                self.groups.append((
                    linear_chunks(pack, oq, qkv_n, H, sms, self.xn, self.qkv, bias=bias),
                    linear_chunks(pack, oo, H, cfg.q_dim, sms, self.attn, self.h, resid=self.h),
                    linear_chunks(pack, og, 2 * I, H, sms, self.xn, self.gu, x_il=self.xn_il),
                    linear_chunks(pack, od, H, I, sms, self.act, self.h, resid=self.h, x_il=self.act_il)))
        ol, _ = offs["lm_head"]
        if world > 1:
            self.head = [GatheredLinear(pack, ol, V, H, sms, self.xn, self.peers, 3, world, rank,
                                        x_il=self.xn_il)]
        else:
            self.head = linear_chunks(pack, ol, V, H, sms, self.xn, self.logits, x_il=self.xn_il)
        P4 = _lib._PTR4
        self._emb = P4(*[extras.embed[k].data_ptr() for k in range(4)])
        self._in_norm = [P4(*[extras.in_norm[l, k].data_ptr() for k in range(4)]) for l in range(cfg.layers)]
        self._post_norm = [P4(*[extras.post_norm[l, k].data_ptr() for k in range(4)]) for l in range(cfg.layers)]
        self._final = P4(*[extras.final_norm[k].data_ptr() for k in range(4)])
        self._kc = [P4(*[t[k].data_ptr() for k in range(4)]) for t in self.kc]
        self._vc = [P4(*[t[k].data_ptr() for k in range(4)]) for t in self.vc]
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        self.graph = None

    def launches_per_step(self) -> int:
        n = lambda g: len(g.calls) if isinstance(g, GatheredLinear) else 1
        return 2 + self.cfg.layers * 4 + sum(n(g) for grp in self.groups for c in grp for g in c) + \
            sum(n(g) for g in self.head) + (1 if self.peers is not None else 0)   # + the logits wait

    def close(self) -> None:
        """Unmap the peers' buffers (collective over the process group)."""
        if self.peers is not None:
            self.peers.close()
            self.peers = None

    def _wait(self, b: int):
        """Arguments of the in-kernel wait for gathered buffer b (none on one GPU)."""
        if self.peers is None:
            return (None, 0, None, None)
        p = self.peers
        return (p.local_flags(b), p.world, p.epoch_ptr(b), p.status.data_ptr())

    def _run(self, s) -> None:
        """Enqueue one step on stream handle s (tokens and pos already set).
        With several GPUs, the kernel that reads a gathered buffer (qkv: 0,
        h: 1, gate_up: 2) first waits for every rank's launches into it; the
        logits (3) get a wait launch of their own at the end of the step."""
        L, cfg, c = self.lib, self.cfg, _lib.check
        H, I = cfg.hidden, cfg.inter
        c(L.pp_embed_rows(self.tokens.data_ptr(), self._emb, cfg.vocab, H, self.h.data_ptr(), H,
                          self.status.data_ptr(), s))
        run = lambda chunks: [g(s) for g in chunks]
        none = (None, 0, None, None)
        for l, (g_qkv, g_o, g_gu, g_d) in enumerate(self.groups):
            c(L.pp_rmsnorm_rows(self.h.data_ptr(), H, self._in_norm[l], H, cfg.rms_eps, self.xn.data_ptr(), H,
                                None, *(self._wait(1) if l > 0 else none), s))
            run(g_qkv)
            c(L.pp_decode_attention(self.qkv.data_ptr(), self.qkv.stride(0), cfg.q_heads, cfg.kv_heads,
                                    cfg.head_dim, self.cos.data_ptr(), self.sin.data_ptr(), self._kc[l],
                                    self._vc[l], cfg.max_pos, self.pos.data_ptr(), self.scale, self.attn.data_ptr(),
                                    self.attn.stride(0), None, self.splits,
                                    self.attn_ws.data_ptr(),
                                    self.attn_ws.numel(), self.status.data_ptr(), *self._wait(0), s))
            run(g_o)
            c(L.pp_rmsnorm_rows(self.h.data_ptr(), H, self._post_norm[l], H, cfg.rms_eps, self.xn.data_ptr(), H,
                                self.xn_il.data_ptr(), *self._wait(1), s))
            run(g_gu)
            c(L.pp_swiglu_rows(self.gu.data_ptr(), self.gu.stride(0), I, self.act.data_ptr(), I,
                               self.act_il.data_ptr(), *self._wait(2), s))
            run(g_d)
        c(L.pp_rmsnorm_rows(self.h.data_ptr(), H, self._final, H, cfg.rms_eps, self.xn.data_ptr(), H,
                            self.xn_il.data_ptr(), *self._wait(1), s))
        run(self.head)
        if self.peers is not None:
            self.peers.wait(3, s)

    def _advance(self) -> None:
        self.pos.add_(1)

    def step(self, tokens=None) -> torch.Tensor:
        """One token per model; returns the logits buffer ``[4][vocab]``."""
        if tokens is not None:
            self.tokens.copy_(torch.as_tensor(tokens, dtype=torch.int32), non_blocking=True)
        if self.graph is not None:
            self.graph.replay()
        else:
            self._run(_lib.stream_handle(self.device))
            self._advance()
        return self.logits

    def capture(self, stream: torch.cuda.Stream) -> None:
        """Capture one step (kernels + position advance) as a CUDA graph; the
        decoder state (position, caches) is unchanged by the capture."""
        pos0 = self.pos.clone()
        with torch.cuda.stream(stream):
            self._run(stream.cuda_stream)       # warm-up outside the graph (argument caches)
            self._advance()
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            self._run(stream.cuda_stream)
            self._advance()
        self.pos.copy_(pos0)
        torch.cuda.synchronize(self.device)
        self.graph = g

    def reset(self) -> None:
        self.pos.zero_()
        self.status.zero_()
