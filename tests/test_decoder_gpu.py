"""Packed Linears inside models (the loader) and the 4-model decoder step.

* ``replace_model_weights_packed`` against the reference's own integration:
  four correlated Qwen2 causal LMs (transformers, random init, a small
  config) have their Linears flattened in ``collect_weights`` order
  (polar_main.py:25-51) and packed by the oracle writer (= the reference
  writer).  The reference path restores the weights (``unpack_quad``,
  quaternion_packer.py:141-214) and writes them into the model as FP16
  (``replace_model_weights``, polar_packer.py:285-316); ours installs
  ``PackedQuadLinear`` modules.  Same prompt, logits within tolerance.
* ``QuadDecoder`` -- one token per model per step, 36-layer-style step
  structure on a 2-layer model -- against a float32 torch restatement of the
  Qwen2 step built from the same restored weights, over several positions
  (KV cache); a captured CUDA graph of the step gives the same logits as the
  eager step, bit for bit.

Tolerance: max|logits - ref| / max|ref| <= 2e-2 per model (FP16 activations
through two decoder layers against float32).
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import formats as of

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _cfg():
    from polar_pack_b200.decoder import DecoderConfig
    return DecoderConfig(layers=2, hidden=512, inter=1024, q_heads=4, kv_heads=2, vocab=1000, max_pos=32)


def _models_flat(cfg, seed):
    """Four correlated flat weight vectors of the cfg's Linears (layer-map order)."""
    from polar_pack_b200.decoder import qwen2_layer_map
    n = sum(e["numel"] for e in qwen2_layer_map(cfg))
    rng = np.random.default_rng(seed)
    base = rng.normal(0, 0.02, n).astype(np.float32)
    out = []
    for _ in range(4):
        w = base + rng.normal(0, 0.002, n).astype(np.float32)
        idx = rng.integers(0, n, n // 1000)
        w[idx] *= 20
        out.append(w.astype(np.float16).astype(np.float32))
    return out


@pytest.fixture(scope="module")
def packed(cuda):
    from polar_pack_b200.quadpack import QuadPackDevice, QuadPackFile
    cfg = _cfg()
    buf = of.pack_quad_bytes(_models_flat(cfg, 0), plug_cap=0.05, threshold_windows=4, window=1_000_000)
    restored = of.unpack_quad_bytes(buf)           # the reference's float restore, per model
    return cfg, buf, restored


def _linear_weights(cfg, restored, k):
    """Model k's Linear weights (float32 of the FP16 the reference installs)."""
    from polar_pack_b200.quadpack import layer_offsets
    from polar_pack_b200.decoder import qwen2_layer_map
    res = {}
    for name, off, (N, K) in layer_offsets(qwen2_layer_map(cfg)):
        res[name] = torch.from_numpy(restored[k][off:off + N * K].reshape(N, K)).half().float()
    return res


def test_replace_model_weights_packed_matches_reference_integration(cuda, packed):
    transformers = pytest.importorskip("transformers")
    from polar_pack_b200.decoder import qwen2_layer_map, replace_model_weights_packed
    from polar_pack_b200.quadpack import QuadPackDevice, QuadPackFile
    cfg, buf, restored = packed
    hf_cfg = transformers.Qwen2Config(vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=cfg.inter,
                                      num_hidden_layers=cfg.layers, num_attention_heads=cfg.q_heads,
                                      num_key_value_heads=cfg.kv_heads, max_position_embeddings=cfg.max_pos,
                                      tie_word_embeddings=False, rms_norm_eps=cfg.rms_eps,
                                      rope_theta=cfg.rope_theta)
    torch.manual_seed(0)
    pk = QuadPackDevice(QuadPackFile(buf), cuda)
    lmap = qwen2_layer_map(cfg)
    prompt = torch.tensor([[3, 17, 256, 999, 42]], device=cuda)
    for k in range(4):
        ref = transformers.Qwen2ForCausalLM(hf_cfg).half().to(cuda).eval()
        ours = transformers.Qwen2ForCausalLM(hf_cfg).half().to(cuda).eval()
        ours.load_state_dict(ref.state_dict())
        names = [n for n, m in ref.named_modules() if isinstance(m, torch.nn.Linear)]
        assert names == [e["name"] for e in lmap]          # the layer map is collect_weights' order
        w = _linear_weights(cfg, restored, k)
        for n, m in ref.named_modules():                    # reference: restored FP16 weights
            if n in w:
                m.weight.data = w[n].half().to(cuda)
        assert replace_model_weights_packed(ours, pk, lmap, k) == len(lmap)
        with torch.no_grad():
            a = ref(prompt).logits.float()
            b = ours(prompt).logits.float()
        err = float((a - b).abs().max() / a.abs().max())
        assert err <= TOL, (k, err)


def _rms(x, w, eps):
    return x * torch.rsqrt((x * x).mean() + eps) * w


def _rope(x, pos, cfg):
    d = cfg.head_dim
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2, dtype=torch.int64).float() / d))
    f = pos * inv
    c, s = torch.cat([f, f]).cos().to(x.device), torch.cat([f, f]).sin().to(x.device)
    rot = torch.cat([-x[..., d // 2:], x[..., :d // 2]], dim=-1)
    return x * c + rot * s


def _ref_step(cfg, W, ex, cache, pos, tok):
    """float32 Qwen2 step of one model (W: its Linear weights, ex: its extras)."""
    hd, nq, nkv = cfg.head_dim, cfg.q_heads, cfg.kv_heads
    h = ex["embed"][tok].float()
    for l in range(cfg.layers):
        p = f"model.layers.{l}."
        x = _rms(h, ex["in_norm"][l], cfg.rms_eps)
        q = W[p + "self_attn.q_proj"] @ x + ex["bias"][l][:cfg.q_dim]
        k = W[p + "self_attn.k_proj"] @ x + ex["bias"][l][cfg.q_dim:cfg.q_dim + cfg.kv_dim]
        v = W[p + "self_attn.v_proj"] @ x + ex["bias"][l][cfg.q_dim + cfg.kv_dim:]
        q = _rope(q.view(nq, hd), pos, cfg)
        k = _rope(k.view(nkv, hd), pos, cfg)
        cache[l][0].append(k)
        cache[l][1].append(v.view(nkv, hd))
        K_ = torch.stack(cache[l][0])                       # [t, nkv, hd]
        V_ = torch.stack(cache[l][1])
        out = []
        for hq in range(nq):
            kvh = hq // (nq // nkv)
            sc = (K_[:, kvh] @ q[hq]) / math.sqrt(hd)
            out.append(torch.softmax(sc, 0) @ V_[:, kvh])
        h = h + W[p + "self_attn.o_proj"] @ torch.cat(out)
        x = _rms(h, ex["post_norm"][l], cfg.rms_eps)
        g, u = W[p + "mlp.gate_proj"] @ x, W[p + "mlp.up_proj"] @ x
        h = h + W[p + "mlp.down_proj"] @ (torch.nn.functional.silu(g) * u)
    return W["lm_head"] @ _rms(h, ex["final"], cfg.rms_eps)


@pytest.fixture(params=[False, True], ids=["serial", "overlap"])
def overlap(request):
    """Launch overlap (programmatic dependent launch) off and on: with it on,
    attention copies cache tiles and the norms read their weights before
    waiting for the previous launch."""
    from polar_pack_b200 import _lib
    old = _lib.set_launch_overlap(request.param)
    yield request.param
    _lib.set_launch_overlap(old)


def test_decoder_step_matches_float32_reference(cuda, packed, overlap):
    from polar_pack_b200.decoder import DecoderExtras, QuadDecoder
    from polar_pack_b200.quadpack import QuadPackDevice, QuadPackFile
    cfg, buf, restored = packed
    pk = QuadPackDevice(QuadPackFile(buf), cuda)
    ex = DecoderExtras.random(cfg, cuda, seed=1)
    dec = QuadDecoder(pk, cfg, ex)
    Ws = [{n: t.to(cuda) for n, t in _linear_weights(cfg, restored, k).items()} for k in range(4)]
    exs = [dict(embed=ex.embed[k].float(), in_norm=ex.in_norm[:, k].float(), post_norm=ex.post_norm[:, k].float(),
                final=ex.final_norm[k].float(), bias=ex.qkv_bias[:, k].float()) for k in range(4)]
    caches = [[([], []) for _ in range(cfg.layers)] for _ in range(4)]
    rng = np.random.default_rng(3)
    steps = []
    for pos in range(6):
        toks = rng.integers(0, cfg.vocab, 4)
        got = dec.step(toks).float().clone()
        steps.append((toks, got))
        for k in range(4):
            ref = _ref_step(cfg, Ws[k], exs[k], caches[k], pos, int(toks[k]))
            err = float((got[k] - ref).abs().max() / ref.abs().max())
            assert err <= TOL, (pos, k, err)
    assert int(dec.status.item()) == 0
    # the captured step replays the same computation
    dec.reset()
    stream = torch.cuda.Stream(cuda)
    dec.capture(stream)
    for toks, got in steps:
        again = dec.step(toks).float()
        torch.cuda.synchronize()
        assert torch.equal(again, got)


def _dec_worker(rank, world, port, buf, q):
    try:
        import os
        import sys
        from datetime import timedelta

        import torch.distributed as dist
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
        from polar_pack_b200.decoder import DecoderExtras, QuadDecoder
        from polar_pack_b200.quadpack import QuadPackDevice, QuadPackFile
        cfg = _cfg()
        pk = QuadPackDevice(QuadPackFile(buf), dev)
        ex = DecoderExtras.random(cfg, dev, seed=1)
        dist_dec = QuadDecoder(pk, cfg, ex, world=world, rank=rank)
        one = QuadDecoder(pk, cfg, ex)
        rng = np.random.default_rng(3)
        worst = 0.0
        for _ in range(4):
            toks = rng.integers(0, cfg.vocab, 4)
            a = dist_dec.step(toks).float().clone()
            b = one.step(toks).float()
            torch.cuda.synchronize(dev)
            worst = max(worst, float((a - b).abs().max() / b.abs().max()))
        ok = worst <= 1e-2 and int(dist_dec.peers.status.item()) == 0
        torch.cuda.synchronize(dev)
        dist_dec.close()
        dist.destroy_process_group()
        q.put((rank, bool(ok), f"{worst:.3g}"))
    except Exception as e:
        q.put((rank, False, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_decoder_two_ranks_matches_one_gpu(packed):
    """Row-sharded decoder on two GPUs (GEMVs gather their rows into both
    ranks' buffers over NVLink) against the one-GPU decoder on the same pack."""
    import socket

    import torch.multiprocessing as mp
    cfg, buf, _ = packed
    with socket.socket() as s_:
        s_.bind(("127.0.0.1", 0))
        port = s_.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_dec_worker, args=(r, 2, port, buf, q)) for r in range(2)]
    for p_ in procs:
        p_.start()
    res = [q.get(timeout=300) for _ in procs]
    for p_ in procs:
        p_.join(timeout=60)
    assert all(ok for _, ok, _ in res), res
