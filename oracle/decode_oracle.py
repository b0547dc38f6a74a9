"""CPU restatement of one batch-1 greedy decode step (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it;
the product never imports it.

It follows the reference's caller of the hot path: scripts/decode_loop.py:
107-124 steps an HF Qwen2 forward per token, every nn.Linear swapped for
W4Linear (decode_loop.py:23-58), then takes the argmax. Here the Qwen2
architecture is written out in fp32 torch ops on the host cores:
  * every int4 linear runs the reference's dequantise-then-matmul path
    (dequantize_v1, kernels.py:50-90, to an fp16 [K, N] copy, then
    x.float() @ W.float(), kernels.py:271-273), restated in C
    (oracle/w4_oracle.c w4o_dequant_matmul, OpenMP over columns), with the
    activation rounded to bf16 on the way in, as W4Linear receives it;
  * RMSNorm, RoPE (rotate-half), GQA attention with exact softmax over the
    growing KV cache, SwiGLU and the residual adds stay in fp32;
  * the tied lm_head is the bf16 embedding widened to fp32.
The weights are copied from a W4DecodeModel (packed words, scales, norms,
bias, embedding), so both sides step the same model.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from . import c_oracle


def _bf16_bits(x: torch.Tensor) -> np.ndarray:
    """fp32 [1, K] -> bf16 bits (round to nearest even), as uint16 numpy."""
    return x.to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16)


class DecodeOracle:
    """fp32 host decoder holding host copies of a W4DecodeModel's weights."""

    def __init__(self, model, threads: int | None = None):
        self.cfg = cfg = model.cfg
        host = lambda t: t.detach().float().cpu()  # noqa: E731
        self.layers = []
        max_kn = 0
        for L in model.layers:
            d = {}
            for name in ("qkv", "o", "gu", "down"):
                p, s = L[name]
                if name == "gu" and getattr(model, "gu_block", 0):
                    # the fused step interleaves gate and up columns; columns are
                    # independent, so the permutation back is exact
                    p = model.deinterleave_gate_up(p, model.gu_block)
                    s = model.deinterleave_gate_up(s, model.gu_block)
                d[name] = (np.ascontiguousarray(p.cpu().numpy()),
                           np.ascontiguousarray(s.cpu().numpy()))
                max_kn = max(max_kn, p.shape[0] * 8 * p.shape[1])
            d["b_qkv"] = host(L["b_qkv"])
            d["in_norm"] = host(L["in_norm"])
            d["post_norm"] = host(L["post_norm"])
            self.layers.append(d)
        self.embed = host(model.embed)
        self.final_norm = host(model.final_norm)
        self.cos, self.sin = host(model.cos), host(model.sin)
        self.wbuf = np.empty((max_kn,), dtype=np.uint16)  # the fp16 weight copy of v1
        self.cores = c_oracle.use_all_cores() if threads is None else c_oracle.lib().w4o_set_threads(threads)
        torch.set_num_threads(self.cores)
        self.reset()

    def reset(self) -> None:
        self.kc = [[] for _ in self.layers]
        self.vc = [[] for _ in self.layers]
        self.pos = 0

    def linear(self, x: torch.Tensor, w) -> torch.Tensor:
        packed, scales = w
        K, N = packed.shape[0] * 8, packed.shape[1]
        y = c_oracle.dequant_matmul(_bf16_bits(x), packed, scales, x_bf16=True,
                                    wbuf=self.wbuf[:K * N].reshape(K, N))
        return torch.from_numpy(y)

    def rms(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        return w * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.cfg.rms_eps))

    @staticmethod
    def rope(x: torch.Tensor, c: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
        half = x.shape[-1] // 2
        return x * c + torch.cat([-x[..., half:], x[..., :half]], -1) * s

    def step(self, token: int) -> torch.Tensor:
        """Runs token at the next position; returns the fp32 logits [vocab]."""
        cfg = self.cfg
        h, kvd, hd = cfg.hidden, cfg.kv_dim, cfg.head_dim
        pos = self.pos
        x = self.embed[token].view(1, h)
        for li, W in enumerate(self.layers):
            r = x
            qkv = self.linear(self.rms(x, W["in_norm"]), W["qkv"]) + W["b_qkv"]
            q = self.rope(qkv[:, :h].view(cfg.heads, hd), self.cos[pos], self.sin[pos])
            k = self.rope(qkv[:, h:h + kvd].view(cfg.kv_heads, hd), self.cos[pos], self.sin[pos])
            v = qkv[:, h + kvd:].view(cfg.kv_heads, hd)
            self.kc[li].append(k)
            self.vc[li].append(v)
            K = torch.stack(self.kc[li], 1)  # [kv, t, hd]
            V = torch.stack(self.vc[li], 1)
            qg = q.view(cfg.kv_heads, cfg.heads // cfg.kv_heads, hd)
            p = torch.softmax(qg @ K.transpose(1, 2) / math.sqrt(hd), -1)
            x = r + self.linear((p @ V).reshape(1, h), W["o"])
            r = x
            gu = self.linear(self.rms(x, W["post_norm"]), W["gu"])
            act = torch.nn.functional.silu(gu[:, :cfg.intermediate]) * gu[:, cfg.intermediate:]
            x = r + self.linear(act, W["down"])
        self.pos += 1
        return (self.rms(x, self.final_norm) @ self.embed.t())[0]


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Rounds float values to the nearest bf16 (ties to even), returned as float64."""
    f = np.asarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((f + 0x7FFF + ((f >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32).astype(np.float64)


def lm_head_logits_f64(h_bits: np.ndarray, norm_bits: np.ndarray, embed_bits: np.ndarray,
                       eps: float, chunk: int = 16384) -> np.ndarray:
    """Logits of the final RMSNorm + tied lm_head in float64, from bf16 bit arrays.

    The normalised row follows the HF Qwen2 bf16 forward the decode loop runs
    (scripts/decode_loop.py:107-124 through the model): x = bf16(bf16(h / rms)
    * w); the logits are embed @ x, summed exactly enough in float64 that only
    the kernel's own fp32 sum and bf16 store differ from them.
    """
    as64 = lambda b: np.asarray(b, dtype=np.uint16).astype(np.uint32).__lshift__(16).view(np.float32).astype(np.float64)  # noqa: E731
    h = as64(h_bits)
    inv = 1.0 / np.sqrt(np.mean(h * h) + eps)
    x = bf16_round(bf16_round(h * inv) * as64(norm_bits))
    out = np.empty((embed_bits.shape[0],), dtype=np.float64)
    for r0 in range(0, embed_bits.shape[0], chunk):
        out[r0:r0 + chunk] = as64(embed_bits[r0:r0 + chunk]) @ x
    return out
