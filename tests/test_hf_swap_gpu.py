"""The drop-in on an HF model: swap_linears on a Qwen2ForCausalLM, then decode.

The reference's caller (scripts/decode_loop.py:61-73, 107-124) swaps every
nn.Linear of an HF Qwen2 model for W4Linear and runs a greedy decode loop
through it. Here a small Qwen2 model is built from a config (no checkpoint)
and copied twice:
  * one copy goes through swap_linears, so every linear (q/k/v with bias, o,
    gate, up, down and the lm_head, which the swap unties from the
    embedding, as in the reference) runs this library's kernels;
  * the other keeps dense fp16 linears whose weights are the oracle's
    dequantisation of the very same packed words.
Both then see a prompt of more than 16 rows (W4Linear's prefill path), a
prompt of at most 16 rows (one fused launch for all rows) and 8 greedy
tokens with the KV cache (one row per call); logits agree within
rtol = atol = 1e-2, and so do the greedy tokens.
"""
import copy

import numpy as np
import pytest
import torch

from oracle import w4_oracle as o

pytestmark = pytest.mark.gpu

from roofline_decoding_b200.linear import W4Linear, swap_linears, weight_bytes_int4  # noqa: E402

DEV = "cuda"


def _models():
    from transformers import Qwen2Config, Qwen2ForCausalLM

    cfg = Qwen2Config(vocab_size=1024, hidden_size=256, intermediate_size=512,
                      num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                      max_position_embeddings=256, tie_word_embeddings=True,
                      attn_implementation="eager")
    torch.manual_seed(0)
    base = Qwen2ForCausalLM(cfg).eval()
    with torch.no_grad():  # HF's init leaves biases at zero: give q/k/v a real bias
        for layer in base.model.layers:
            for proj in (layer.self_attn.q_proj, layer.self_attn.k_proj, layer.self_attn.v_proj):
                proj.bias.normal_(0.0, 0.05)
    w4 = copy.deepcopy(base).to(DEV, torch.float16)
    dense = copy.deepcopy(base).to(DEV, torch.float16)
    names = swap_linears(w4)
    # the dense twin: the oracle's fp16 dequantisation of the same packed words
    mods = dict(w4.named_modules())
    with torch.no_grad():
        for name in names:
            lin = mods[name]
            wq = o.dequantize_fp16(lin.packed.cpu().numpy(), lin.scales.cpu().numpy())  # [K, N]
            parent, _, attr = name.rpartition(".")
            d = dense.get_submodule(parent) if parent else dense
            old = getattr(d, attr)
            new = torch.nn.Linear(old.in_features, old.out_features, bias=old.bias is not None,
                                  device=DEV, dtype=torch.float16)
            new.weight.copy_(torch.from_numpy(np.ascontiguousarray(wq.T)).to(DEV))
            if old.bias is not None:
                new.bias.copy_(old.bias)
            setattr(d, attr, new)
    return base, w4, dense, names


def _close(a, b):
    torch.testing.assert_close(a.float(), b.float(), rtol=1e-2, atol=1e-2)


@torch.no_grad()
def test_swap_linears_qwen2_matches_dequantised_dense_model():
    base, w4, dense, names = _models()
    n_linear = sum(isinstance(m, torch.nn.Linear) for m in base.modules())
    assert len(names) == n_linear == 2 * 7 + 1  # 7 per layer + the lm_head
    assert all(isinstance(m, W4Linear) for n, m in w4.named_modules() if n in names)
    assert w4.model.layers[0].self_attn.q_proj.has_bias
    g = torch.Generator().manual_seed(3)
    for prompt_len in (24, 12):  # > 16 rows: prefill path; <= 16 rows: one fused launch
        ids = torch.randint(0, 1024, (1, prompt_len), generator=g).to(DEV)
        oa = w4(ids, use_cache=True)
        ob = dense(ids, use_cache=True)
        _close(oa.logits, ob.logits)
        cache_a, cache_b = oa.past_key_values, ob.past_key_values
        tok = ob.logits[:, -1].argmax(-1, keepdim=True)
        for step in range(8):  # greedy decode: one row per W4Linear call
            oa = w4(tok, past_key_values=cache_a, use_cache=True)
            ob = dense(tok, past_key_values=cache_b, use_cache=True)
            _close(oa.logits, ob.logits)
            la, lb = oa.logits[0, -1].float(), ob.logits[0, -1].float()
            top2 = torch.topk(lb, 2).values
            if (top2[0] - top2[1]).item() > 2e-2:  # not a near tie
                assert int(la.argmax()) == int(lb.argmax()), (prompt_len, step)
            cache_a, cache_b = oa.past_key_values, ob.past_key_values
            tok = lb.argmax().view(1, 1)


@torch.no_grad()
@pytest.mark.parametrize("n_out", [384, 392])
def test_w4linear_row_paths_with_bias(n_out):
    """One layer through the row paths of W4Linear.forward, with bias: up to 16
    rows in one fused launch, more rows on the tensor-core GEMM (n_out a
    multiple of 128) or dequantise-then-matmul (otherwise)."""
    torch.manual_seed(1)
    lin = torch.nn.Linear(512, n_out, bias=True).to(DEV, torch.float16)
    torch.nn.init.normal_(lin.bias, 0.0, 0.1)
    w4 = W4Linear(lin)
    wq = torch.from_numpy(o.dequantize_fp16(w4.packed.cpu().numpy(),
                                            w4.scales.cpu().numpy())).to(DEV)
    for rows in (1, 5, 16, 17, 40):
        x = torch.randn((rows, 512), device=DEV).half()
        want = ((x.float() @ wq.float()).half() + lin.bias).float()
        _close(w4(x), want)
        _close(w4(x.view(rows, 1, 512)).view(rows, n_out), want)  # [..., K] inputs keep their shape


def test_weight_bytes_int4_matches_the_reference_formula():
    base, w4, _, names = _models()
    # scripts/decode_loop.py:76-85: packed words * 4 + scales * 2 for W4Linear,
    # 2 bytes per parameter for embeddings and dense linears
    want = 0
    for m in w4.modules():
        if isinstance(m, W4Linear):
            K, N = m.in_features, m.out_features
            want += (K // 8) * N * 4 + (K // 128) * N * 2
        elif isinstance(m, torch.nn.Embedding):
            want += m.weight.numel() * 2
    assert weight_bytes_int4(w4) == want
    emb = base.model.embed_tokens.weight.numel() * 2
    lin = sum(m.weight.numel() for n, m in base.named_modules() if isinstance(m, torch.nn.Linear))
    assert want == emb + lin // 2 + lin // 128 * 2  # int4 + one fp16 scale per 128 weights
