"""The decode attention kernel (w4_decode_attention) on its own, against an
fp32 torch restatement of the reference model's step (RoPE in bf16
arithmetic, the new k/v appended to the cache, exact softmax over positions
0..pos, GQA).

Covers both kernel instances (groups up to 8 and up to 16 q heads per KV
head), positions on both sides of the split and tile boundaries, the cache
write of the new position, and the clamping of a position outside the cache.
Bars: the output within bf16 rounding (rtol 2^-7, atol 2e-3 on O(1) values);
the cache row of the new position bit-exact.
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from roofline_decoding_b200 import _lib  # noqa: E402
from roofline_decoding_b200.kernels import _stream_ptr  # noqa: E402

HD = 128
DEV = "cuda"


def rbf(x):
    return x.to(torch.bfloat16).float()


def rope_tables(max_seq, theta=1e6):
    inv = 1.0 / (theta ** (torch.arange(0, HD, 2, device=DEV).float() / HD))
    f = torch.outer(torch.arange(max_seq, device=DEV).float(), inv)
    emb = torch.cat([f, f], -1)
    return emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)


def rope_bf16(x, c, s):
    """round(round(x*cos) + round(rot(x)*sin)) per element, as the kernel."""
    rot = torch.cat([-x[..., HD // 2:], x[..., :HD // 2]], -1)
    return rbf(rbf(x * c) + rbf(rot * s))


def run_case(heads, kv, pos, max_seq, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    cos, sin = rope_tables(max_seq)
    qkv = torch.randn((heads + 2 * kv) * HD, generator=g, device=DEV).to(torch.bfloat16)
    kc = torch.randn((kv, max_seq, HD), generator=g, device=DEV).to(torch.bfloat16)
    vc = torch.randn((kv, max_seq, HD), generator=g, device=DEV).to(torch.bfloat16)
    kc0, vc0 = kc.clone(), vc.clone()
    out = torch.empty(heads * HD, device=DEV, dtype=torch.bfloat16)
    pos_t = torch.tensor([pos], device=DEV, dtype=torch.int64)
    _lib.check(_lib.load().w4_decode_attention(
        qkv.data_ptr(), cos.data_ptr(), sin.data_ptr(), pos_t.data_ptr(), kc.data_ptr(),
        vc.data_ptr(), out.data_ptr(), heads, kv, HD, max_seq, 0, _stream_ptr(qkv.device)),
        "w4_decode_attention")
    torch.cuda.synchronize()
    p = min(max(pos, 0), max_seq - 1)
    c, s = cos[p].float(), sin[p].float()
    x = qkv.float()
    q = rope_bf16(x[:heads * HD].view(heads, HD), c, s)
    k = rope_bf16(x[heads * HD:(heads + kv) * HD].view(kv, HD), c, s)
    v = x[(heads + kv) * HD:].view(kv, HD)
    K = kc0.float().clone()
    V = vc0.float().clone()
    K[:, p] = k
    V[:, p] = v
    G = heads // kv
    want = torch.empty(heads, HD, device=DEV)
    for h in range(heads):
        kvh = h // G
        sc = (K[kvh, :p + 1] @ q[h]) / math.sqrt(HD)
        want[h] = torch.softmax(sc, 0) @ V[kvh, :p + 1]
    # the new position's row is written to the cache, nothing else changes
    assert torch.equal(kc[:, p], k.to(torch.bfloat16))
    assert torch.equal(vc[:, p], v.to(torch.bfloat16))
    keep = torch.ones(max_seq, dtype=torch.bool, device=DEV)
    keep[p] = False
    assert torch.equal(kc[:, keep], kc0[:, keep]) and torch.equal(vc[:, keep], vc0[:, keep])
    torch.testing.assert_close(out.float().view(heads, HD), want, rtol=2 ** -7, atol=2e-3)


@pytest.mark.parametrize("heads,kv", [(2, 2), (4, 2), (12, 2), (16, 2), (24, 2), (32, 2),
                                      (16, 1), (8, 4)])
def test_attention_groups(heads, kv):
    """Groups 1, 2, 6, 8 (the 8-head instance) and 12, 16 (the 16-head instance)."""
    run_case(heads, kv, pos=200, max_seq=512, seed=heads * 10 + kv)


@pytest.mark.parametrize("pos", [0, 1, 7, 8, 9, 63, 64, 65, 511, 512, 513, 700, 1023])
def test_attention_positions(pos):
    """Split (8) and tile (64 rows) boundaries, up to a full cache."""
    run_case(12, 2, pos=pos, max_seq=1024, seed=pos)


def test_attention_position_outside_cache_is_clamped():
    run_case(12, 2, pos=5000, max_seq=256, seed=1)
    run_case(12, 2, pos=-3, max_seq=256, seed=2)
