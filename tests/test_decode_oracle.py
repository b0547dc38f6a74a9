"""The CPU decode oracle (oracle/decode_oracle.py) on a tiny Qwen2-architecture model.

The oracle steps the model with the reference's dequantise-then-matmul path
in C for every int4 linear; here it is checked on the CPU against a plain
fp32 restatement that dequantises with numpy, so that the oracle the GPU
decode tests and the bench's CPU baseline use is itself pinned.
"""
import math
from types import SimpleNamespace

import numpy as np
import torch

from oracle import w4_oracle as o
from oracle.decode_oracle import DecodeOracle
from roofline_decoding_b200.decode import DecodeConfig

TINY = DecodeConfig(hidden=256, layers=2, heads=2, kv_heads=1, intermediate=512, vocab=300,
                    max_seq=32, name="tiny")


def _tiny_model(seed=0):
    rng = np.random.default_rng(seed)
    cfg = TINY
    h, kv, inter = cfg.hidden, cfg.kv_dim, cfg.intermediate
    shapes = {"qkv": (h, h + 2 * kv), "o": (h, h), "gu": (h, 2 * inter), "down": (inter, h)}
    bf = lambda a: torch.from_numpy(a.astype(np.float32)).to(torch.bfloat16)  # noqa: E731
    layers = []
    for _ in range(cfg.layers):
        L = {}
        for name, (K, N) in shapes.items():
            p, s = o.pack_weights((rng.standard_normal((K, N)) * 0.08).astype(np.float16))
            L[name] = (torch.from_numpy(p), torch.from_numpy(s))
        L["b_qkv"] = bf(rng.standard_normal(h + 2 * kv) * 0.02)
        L["in_norm"] = bf(1 + 0.05 * rng.standard_normal(h))
        L["post_norm"] = bf(1 + 0.05 * rng.standard_normal(h))
        layers.append(L)
    inv = 1.0 / (cfg.rope_theta ** (np.arange(0, cfg.head_dim, 2) / cfg.head_dim))
    freqs = np.outer(np.arange(cfg.max_seq), inv)
    emb = np.concatenate([freqs, freqs], -1)
    return SimpleNamespace(cfg=cfg, layers=layers, embed=bf(rng.standard_normal((cfg.vocab, h)) * 0.08),
                           final_norm=bf(1 + 0.05 * rng.standard_normal(h)), cos=bf(np.cos(emb)),
                           sin=bf(np.sin(emb)))


def _plain_logits(model, ids):
    """fp32 forward with numpy-dequantised weights, one token at a time."""
    cfg = model.cfg
    f = lambda t: t.float()  # noqa: E731
    deq = lambda ps: torch.from_numpy(o.dequantize_f32(ps[0].numpy(), ps[1].numpy()))  # noqa: E731
    Ls = [{k: deq(v) if isinstance(v, tuple) else f(v) for k, v in L.items()} for L in model.layers]
    rms = lambda x, w: w * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + cfg.rms_eps))  # noqa: E731
    h, kvd, hd = cfg.hidden, cfg.kv_dim, cfg.head_dim
    kc, vc, out = [[] for _ in Ls], [[] for _ in Ls], []
    cos, sin, embed = f(model.cos), f(model.sin), f(model.embed)
    for pos, tok in enumerate(ids):
        x = embed[tok].view(1, h)
        for li, W in enumerate(Ls):
            r = x
            qkv = rms(x, W["in_norm"]) @ W["qkv"] + W["b_qkv"]
            rot = lambda t: t * cos[pos] + torch.cat([-t[..., hd // 2:], t[..., :hd // 2]], -1) * sin[pos]  # noqa: E731
            q = rot(qkv[:, :h].view(cfg.heads, hd))
            kc[li].append(rot(qkv[:, h:h + kvd].view(cfg.kv_heads, hd)))
            vc[li].append(qkv[:, h + kvd:].view(cfg.kv_heads, hd))
            K, V = torch.stack(kc[li], 1), torch.stack(vc[li], 1)
            qg = q.view(cfg.kv_heads, cfg.heads // cfg.kv_heads, hd)
            a = (torch.softmax(qg @ K.transpose(1, 2) / math.sqrt(hd), -1) @ V).reshape(1, h)
            x = r + a @ W["o"]
            r = x
            gu = rms(x, W["post_norm"]) @ W["gu"]
            x = r + (torch.nn.functional.silu(gu[:, :cfg.intermediate]) * gu[:, cfg.intermediate:]) @ W["down"]
        out.append((rms(x, f(model.final_norm)) @ embed.t())[0])
    return out


def test_decode_oracle_matches_plain_fp32_forward():
    model = _tiny_model()
    ids = [5, 17, 250, 3, 99, 42]
    want = _plain_logits(model, ids)
    ref = DecodeOracle(model, threads=2)
    for i, tok in enumerate(ids):
        got = ref.step(tok)
        scale = want[i].abs().max().item()
        # the oracle rounds each linear's input to bf16 and its weights to fp16
        assert (got - want[i]).abs().max().item() < 0.02 * scale, f"step {i}"
    assert ref.pos == len(ids)
    ref.reset()
    assert ref.pos == 0 and torch.equal(ref.step(ids[0]), DecodeOracle(model, threads=2).step(ids[0]))
