"""Batch-1 greedy decode of a Qwen2-architecture model with W4A16 linears, one CUDA graph per step.

Replaces the caller of the hot path in scripts/decode_loop.py:106-124 (HF
forward with a dynamic cache, `.item()` per token): the step here has a
static KV cache, keeps the token on the device, and is captured once into a
CUDA graph, so a decoded token costs one graph replay and no host sync.

Architecture (Qwen2.5-1.5B by default): RMSNorm, q/k/v with bias, RoPE
(theta 1e6, rotate-half), GQA attention, o-proj, SwiGLU MLP, tied bf16
embedding / lm_head, greedy argmax. Every decoder linear is int4 (group 128,
the reference's packing); q|k|v and gate|up are packed as one matrix each
(columns are independent, so the concatenation is exact) and run as one
fused GEMV. Weights are random (seeded): there is no checkpoint here.

Precision follows HF's bf16 Qwen2 path: RMSNorm in fp32 rounded to bf16 and
scaled by the bf16 weight, RoPE in bf16, attention softmax in fp32, SiLU and
the gate*up product in bf16, residual adds in bf16.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import GemvConfig
from .kernels import fused_launch, pack_weights, tuned_config, w4_matmul
from .roofline import decode_step_bytes


@dataclass
class DecodeConfig:
    hidden: int = 1536
    layers: int = 28
    heads: int = 12
    kv_heads: int = 2
    intermediate: int = 8960
    vocab: int = 151936
    rope_theta: float = 1e6
    rms_eps: float = 1e-6
    max_seq: int = 2048
    name: str = "Qwen2.5-1.5B (random init)"

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @property
    def kv_dim(self) -> int:
        return self.head_dim * self.kv_heads

    def as_roofline_dict(self) -> dict:
        return {"name": self.name, "hidden": self.hidden, "layers": self.layers,
                "heads": self.heads, "kv_heads": self.kv_heads,
                "intermediate": self.intermediate, "vocab": self.vocab,
                "tied_embeddings": True}


QWEN25_15B = DecodeConfig()


@dataclass
class DenseLayer:
    """Dense (unquantised) weights of one layer, [in, out] layout, for references."""
    w_qkv: torch.Tensor
    b_qkv: torch.Tensor
    w_o: torch.Tensor
    w_gu: torch.Tensor
    w_down: torch.Tensor
    in_norm: torch.Tensor
    post_norm: torch.Tensor


def _rand(shape, gen, device, std):
    return (torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std)


class W4DecodeModel:
    """Static-KV, graph-captured batch-1 greedy decoder with int4 linears."""

    MODES = ("mega", "fused", "torch")
    # The fused step's gate|up GEMV tile: the SwiGLU epilogue pairs the first and
    # second half of a tile, so gate and up alternate in blocks of half a tile.
    GU_CONFIG = (2, 4, 2, 1, 0)
    GU_BLOCK = 16 * GU_CONFIG[0]
    # Tiles of the fused step's other GEMVs, keyed by (K, N), chosen by timing
    # whole captured steps of the Qwen2.5-1.5B architecture (bf16): inside a
    # step they share the SMs with the kernels around them, and the tile that
    # wins a chain of the GEMV alone can lose there (o: (1, 4, 3) took the step
    # from 0.721 to 0.766 ms). Other shapes use the tuned tile.
    STEP_TILES = {(1536, 2048): (1, 8, 2, 1, 0), (1536, 1536): (1, 8, 2, 1, 0),
                  (8960, 1536): (1, 8, 2, 8, 0)}

    @staticmethod
    def interleave_gate_up(w: torch.Tensor, block: int) -> torch.Tensor:
        """[..., gate | up] columns -> alternating blocks: gate 0..b-1, up 0..b-1, gate b.."""
        *lead, n2 = w.shape
        inter = n2 // 2
        g = w[..., :inter].reshape(*lead, inter // block, 1, block)
        u = w[..., inter:].reshape(*lead, inter // block, 1, block)
        return torch.cat([g, u], dim=-2).reshape(*lead, n2)

    @staticmethod
    def deinterleave_gate_up(w: torch.Tensor, block: int) -> torch.Tensor:
        """The inverse of interleave_gate_up: alternating blocks -> [gate | up]."""
        *lead, n2 = w.shape
        v = w.reshape(*lead, n2 // (2 * block), 2, block)
        return torch.cat([v[..., 0, :].reshape(*lead, n2 // 2),
                          v[..., 1, :].reshape(*lead, n2 // 2)], dim=-1)

    def __init__(self, cfg: DecodeConfig = QWEN25_15B, device: str | torch.device = "cuda",
                 seed: int = 0, std: float = 0.02, keep_dense: bool = False, fused: bool = True,
                 mode: str | None = None):
        """mode: "mega" (the step as one persistent kernel, w4_decode_step), "fused"
        (142 PDL-chained kernels) or "torch" (torch ops around the fused GEMVs);
        without it, `fused` picks "fused" or "torch"."""
        self.cfg = cfg
        self.mode = mode or ("fused" if fused else "torch")
        if self.mode not in self.MODES:
            raise ValueError(f"mode must be one of {self.MODES}, got {self.mode!r}")
        self.fused = self.mode != "torch"
        self.device = torch.device(device)
        self.dtype = torch.bfloat16
        gen = torch.Generator(device=self.device).manual_seed(seed)
        h, kv, inter = cfg.hidden, cfg.kv_dim, cfg.intermediate
        bf = self.dtype
        nl = cfg.layers
        # int4 weights stacked over layers ([layers * K/8, N] / [layers * K/128, N]);
        # each layer uses row views of them
        shapes = {"qkv": (h, h + 2 * kv), "o": (h, h), "gu": (h, 2 * inter), "down": (inter, h)}
        self.w4 = {k: (torch.empty((nl * K // 8, N), dtype=torch.int32, device=self.device),
                       torch.empty((nl * K // 128, N), dtype=torch.float16, device=self.device))
                   for k, (K, N) in shapes.items()}
        self.b_qkv = torch.empty((nl, h + 2 * kv), dtype=bf, device=self.device)
        self.in_norms = torch.empty((nl, h), dtype=bf, device=self.device)
        self.post_norms = torch.empty((nl, h), dtype=bf, device=self.device)
        self.layers = []
        self.dense: list[DenseLayer] | None = [] if keep_dense else None
        # The fused step computes SwiGLU in the gate|up GEMV's epilogue: there the
        # gate and up columns alternate in blocks of GU_BLOCK, so that one CTA
        # holds matching gate and up outputs. Columns are independent, so the
        # permutation is exact; the other modes keep [gate | up].
        self.gu_block = self.GU_BLOCK if self.mode == "fused" else 0
        for li in range(nl):
            w_qkv = _rand((h, h + 2 * kv), gen, self.device, std).half()
            w_o = _rand((h, h), gen, self.device, std).half()
            w_gu = _rand((h, 2 * inter), gen, self.device, std).half()
            w_down = _rand((inter, h), gen, self.device, std).half()
            layer = {}
            w_gu_packed = self.interleave_gate_up(w_gu, self.gu_block) if self.gu_block else w_gu
            for name, w in (("qkv", w_qkv), ("o", w_o), ("gu", w_gu_packed), ("down", w_down)):
                K = shapes[name][0]
                pk, sc = pack_weights(w)
                dp = self.w4[name][0][li * K // 8:(li + 1) * K // 8]
                ds = self.w4[name][1][li * K // 128:(li + 1) * K // 128]
                dp.copy_(pk)
                ds.copy_(sc)
                layer[name] = (dp, ds)
            self.b_qkv[li].copy_(_rand((h + 2 * kv,), gen, self.device, 0.02).to(bf))
            self.in_norms[li].copy_((1.0 + _rand((h,), gen, self.device, 0.05)).to(bf))
            self.post_norms[li].copy_((1.0 + _rand((h,), gen, self.device, 0.05)).to(bf))
            layer["b_qkv"] = self.b_qkv[li]
            layer["in_norm"] = self.in_norms[li]
            layer["post_norm"] = self.post_norms[li]
            self.layers.append(layer)
            if keep_dense:
                self.dense.append(DenseLayer(w_qkv, layer["b_qkv"], w_o, w_gu, w_down,
                                             layer["in_norm"], layer["post_norm"]))
        self.embed = _rand((cfg.vocab, h), gen, self.device, std).to(bf)  # tied lm_head
        self.final_norm = (1.0 + _rand((h,), gen, self.device, 0.05)).to(bf)
        # RoPE tables (rotate-half layout), computed in fp32 like HF and cast per use
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, cfg.head_dim, 2, device=self.device,
                                                         dtype=torch.float32) / cfg.head_dim))
        t = torch.arange(cfg.max_seq, device=self.device, dtype=torch.float32)
        freqs = torch.outer(t, inv)
        emb = torch.cat([freqs, freqs], dim=-1)
        self.cos = emb.cos().to(bf)
        self.sin = emb.sin().to(bf)
        self.k_cache = torch.zeros((cfg.layers, cfg.kv_heads, cfg.max_seq, cfg.head_dim),
                                   dtype=bf, device=self.device)
        self.v_cache = torch.zeros_like(self.k_cache)
        # step state (device-resident): current token, position, prompt
        self.token = torch.zeros((1,), dtype=torch.long, device=self.device)
        self.pos = torch.zeros((1,), dtype=torch.long, device=self.device)
        self.prompt = torch.zeros((cfg.max_seq,), dtype=torch.long, device=self.device)
        self.prompt_len = torch.zeros((1,), dtype=torch.long, device=self.device)
        self.positions = torch.arange(cfg.max_seq, device=self.device)
        self.logits = torch.empty((1, cfg.vocab), dtype=bf, device=self.device)
        self.graph: torch.cuda.CUDAGraph | None = None
        self.pdl = True
        # activation buffers of the fused step (device-resident, graph-stable)
        self.h = torch.zeros((1, h), dtype=bf, device=self.device)
        self.qkv_buf = torch.empty((1, h + 2 * kv), dtype=bf, device=self.device)
        self.attn_buf = torch.empty((1, h), dtype=bf, device=self.device)
        # the fused step's gate|up GEMV writes silu(gate) * up; the others write gate | up
        self.gu_buf = torch.empty((1, inter if self.gu_block else 2 * inter), dtype=bf,
                                  device=self.device)
        self.ws = torch.zeros((int(_lib.load().w4_lm_head_workspace_bytes()),), dtype=torch.uint8,
                              device=self.device)
        self._cfgs: dict | None = None
        self._desc: _lib.DecodeModel | None = None
        self.scratch: torch.Tensor | None = None
        if self.mode == "mega":
            self._init_mega()

    def _init_mega(self) -> None:
        """The w4_decode_model descriptor and the step's scratch."""
        cfg = self.cfg
        d = _lib.DecodeModel()
        d.layers, d.hidden, d.intermediate = cfg.layers, cfg.hidden, cfg.intermediate
        d.heads, d.kv_heads, d.head_dim = cfg.heads, cfg.kv_heads, cfg.head_dim
        d.vocab, d.max_seq, d.eps = cfg.vocab, cfg.max_seq, cfg.rms_eps
        for name in ("qkv", "o", "gu", "down"):
            setattr(d, f"{name}_packed", self.w4[name][0].data_ptr())
            setattr(d, f"{name}_scales", self.w4[name][1].data_ptr())
        d.qkv_bias, d.in_norm = self.b_qkv.data_ptr(), self.in_norms.data_ptr()
        d.post_norm, d.final_norm = self.post_norms.data_ptr(), self.final_norm.data_ptr()
        d.embed, d.cos_table, d.sin_table = (self.embed.data_ptr(), self.cos.data_ptr(),
                                             self.sin.data_ptr())
        d.k_cache, d.v_cache = self.k_cache.data_ptr(), self.v_cache.data_ptr()
        d.prompt, d.prompt_len = self.prompt.data_ptr(), self.prompt_len.data_ptr()
        d.token, d.pos, d.logits = (self.token.data_ptr(), self.pos.data_ptr(),
                                    self.logits.data_ptr())
        lib = _lib.load()
        n = ctypes.c_size_t(0)
        with torch.cuda.device(self.device):
            _lib.check(lib.w4_decode_step_scratch_bytes(ctypes.byref(d), ctypes.byref(n)),
                       "w4_decode_step_scratch_bytes")
        self._desc = d
        self.scratch = torch.zeros((int(n.value),), dtype=torch.uint8, device=self.device)

    # ---------------------------------------------------------------- ops
    def rmsnorm(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        xf = x.float()
        xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.cfg.rms_eps)
        return w * xf.to(self.dtype)

    def rope(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        half = x.shape[-1] // 2
        rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
        return x * cos + rot * sin

    def linear(self, x: torch.Tensor, name: str, layer: dict) -> torch.Tensor:
        p, s = layer[name]
        return w4_matmul(x, p, s, out_dtype=self.dtype, pdl=self.pdl)

    def attention(self, li: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        """GQA decode attention over the static cache, positions <= pos."""
        cfg = self.cfg
        kc, vc = self.k_cache[li], self.v_cache[li]
        kc.index_copy_(1, self.pos, k.view(cfg.kv_heads, 1, cfg.head_dim))
        vc.index_copy_(1, self.pos, v.view(cfg.kv_heads, 1, cfg.head_dim))
        mask = (self.positions <= self.pos).view(1, 1, 1, -1)
        o = torch.nn.functional.scaled_dot_product_attention(
            q.view(1, cfg.heads, 1, cfg.head_dim), kc.unsqueeze(0), vc.unsqueeze(0),
            attn_mask=mask, scale=1.0 / math.sqrt(cfg.head_dim), enable_gqa=True)
        return o.reshape(1, cfg.hidden)

    def forward_token(self) -> None:
        """One decode step on the device state (capturable: no host syncs)."""
        with torch.cuda.nvtx.range("w4_decode_step"):  # lets a profiler select one step
            if self.mode == "mega":
                self._forward_mega()
            elif self.mode == "fused":
                self._forward_fused()
            else:
                self._forward_torch()

    def _forward_mega(self) -> None:
        """The step as one cooperative launch of libw4b200.so (w4_decode_step)."""
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(_lib.load().w4_decode_step(ctypes.byref(self._desc), self.scratch.data_ptr(),
                                              self.scratch.numel(), stream), "w4_decode_step")

    def _gemv_cfgs(self) -> dict:
        if self._cfgs is None:
            cfg, bf = self.cfg, self.dtype
            shapes = {"qkv": (cfg.hidden, cfg.hidden + 2 * cfg.kv_dim), "o": (cfg.hidden, cfg.hidden),
                      "gu": (cfg.hidden, 2 * cfg.intermediate), "down": (cfg.intermediate, cfg.hidden)}
            out = {}
            for name, (K, N) in shapes.items():
                c = tuned_config(1, K, N, bf, bf, None, None, self.device,
                                 streaming=self.mode != "fused")
                if self.mode == "fused" and (K, N) in self.STEP_TILES:
                    c = GemvConfig(*self.STEP_TILES[(K, N)])
                if name == "gu" and self.gu_block:
                    c = GemvConfig(*self.GU_CONFIG)  # the tile the columns are interleaved for
                out[name] = c.with_pdl(1 if self.pdl else 0)
            self._cfgs = out
        return self._cfgs

    def _forward_fused(self) -> None:
        """The step as 1 + 5 * layers + 1 kernels of libw4b200.so (PDL-chained)."""
        cfg, lib = self.cfg, _lib.load()
        cfgs = self._gemv_cfgs()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        pdl = 1 if self.pdl else 0
        chk = _lib.check
        chk(lib.w4_decode_embed(self.embed.data_ptr(), cfg.vocab, cfg.hidden,
                                self.prompt.data_ptr(), self.prompt_len.data_ptr(),
                                self.token.data_ptr(), self.pos.data_ptr(), self.h.data_ptr(),
                                pdl, stream), "w4_decode_embed")
        for li, L in enumerate(self.layers):
            fused_launch(self.h, *L["qkv"], self.qkv_buf, cfgs["qkv"], _lib.W4_PRO_RMSNORM,
                         L["in_norm"], cfg.rms_eps, _lib.W4_EPI_BIAS, L["b_qkv"])
            chk(lib.w4_decode_attention(self.qkv_buf.data_ptr(), self.cos.data_ptr(),
                                        self.sin.data_ptr(), self.pos.data_ptr(),
                                        self.k_cache[li].data_ptr(), self.v_cache[li].data_ptr(),
                                        self.attn_buf.data_ptr(), cfg.heads, cfg.kv_heads,
                                        cfg.head_dim, cfg.max_seq, pdl, stream),
                "w4_decode_attention")
            fused_launch(self.attn_buf, *L["o"], self.h, cfgs["o"],
                         epilogue=_lib.W4_EPI_RESIDUAL, epi_src=self.h)
            # gate|up with SwiGLU in its epilogue (interleaved columns), then the
            # down projection on the activation, residual added in its epilogue
            fused_launch(self.h, *L["gu"], self.gu_buf, cfgs["gu"], _lib.W4_PRO_RMSNORM,
                         L["post_norm"], cfg.rms_eps, _lib.W4_EPI_SWIGLU)
            fused_launch(self.gu_buf, *L["down"], self.h, cfgs["down"],
                         epilogue=_lib.W4_EPI_RESIDUAL, epi_src=self.h)
        chk(lib.w4_lm_head_argmax(self.h.data_ptr(), self.final_norm.data_ptr(), cfg.rms_eps,
                                  self.embed.data_ptr(), cfg.vocab, cfg.hidden,
                                  self.logits.data_ptr(), self.token.data_ptr(),
                                  self.pos.data_ptr(), self.ws.data_ptr(), self.ws.numel(), pdl,
                                  stream), "w4_lm_head_argmax")

    def _forward_torch(self) -> None:
        """The same step with torch ops around the fused GEMVs (reference path)."""
        cfg = self.cfg
        is_prompt = self.pos < self.prompt_len
        tok = torch.where(is_prompt, self.prompt.index_select(0, self.pos), self.token)
        x = self.embed.index_select(0, tok)  # [1, h]
        cos = self.cos.index_select(0, self.pos)
        sin = self.sin.index_select(0, self.pos)
        h, kvd = cfg.hidden, cfg.kv_dim
        for li, L in enumerate(self.layers):
            r = x
            xn = self.rmsnorm(x, L["in_norm"])
            qkv = self.linear(xn, "qkv", L) + L["b_qkv"]
            q = self.rope(qkv[:, :h].view(cfg.heads, cfg.head_dim), cos, sin)
            k = self.rope(qkv[:, h:h + kvd].view(cfg.kv_heads, cfg.head_dim), cos, sin)
            v = qkv[:, h + kvd:]
            a = self.attention(li, q, k, v)
            x = r + self.linear(a, "o", L)
            r = x
            xn = self.rmsnorm(x, L["post_norm"])
            gu = self.linear(xn, "gu", L)
            act = torch.nn.functional.silu(gu[:, :cfg.intermediate]) * gu[:, cfg.intermediate:]
            x = r + self.linear(act, "down", L)
        xn = self.rmsnorm(x, self.final_norm)
        torch.matmul(xn, self.embed.t(), out=self.logits)
        self.token.copy_(torch.argmax(self.logits, dim=-1))
        self.pos.add_(1)

    # ---------------------------------------------------------------- driver
    def tune(self) -> None:
        """Tunes (or loads) every GEMV tile; must run before capture."""
        if self.mode != "mega":
            self._gemv_cfgs()

    def launches_per_step(self) -> int:
        """Kernels of libw4b200.so one step launches."""
        return 1 if self.mode == "mega" else 2 + 5 * self.cfg.layers

    def set_prompt(self, ids: torch.Tensor) -> None:
        n = ids.numel()
        self.prompt[:n].copy_(ids.to(self.device).view(-1))
        self.prompt_len.fill_(n)
        self.pos.zero_()
        self.token.zero_()
        self.k_cache.zero_()
        self.v_cache.zero_()

    def capture(self) -> None:
        self.tune()
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        saved = (self.pos.clone(), self.token.clone())
        with torch.cuda.stream(s):
            for _ in range(2):  # warm up outside capture
                self.forward_token()
        torch.cuda.current_stream(self.device).wait_stream(s)
        self.pos.copy_(saved[0])
        self.token.copy_(saved[1])
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.forward_token()
        # capture does not execute: restore the state and reset the cache
        self.pos.copy_(saved[0])
        self.token.copy_(saved[1])

    def step(self) -> None:
        if self.graph is None:
            self.capture()
        self.graph.replay()

    def generate(self, prompt_ids: torch.Tensor, new_tokens: int) -> torch.Tensor:
        """Greedy decode; returns the generated ids (one host sync at the end)."""
        if self.graph is None:
            self.capture()
        self.set_prompt(prompt_ids)
        out = torch.empty((new_tokens,), dtype=torch.long, device=self.device)
        n_prompt = prompt_ids.numel()
        for _ in range(n_prompt):
            self.graph.replay()
        for i in range(new_tokens):
            out[i:i + 1].copy_(self.token)
            self.graph.replay()
        return out

    def bytes_per_step(self, seq_len: int | None = None) -> int:
        """HBM bytes one step reads (the attention reads the whole static cache)."""
        return decode_step_bytes(self.cfg.as_roofline_dict(),
                                 seq_len=seq_len or self.cfg.max_seq)["total"]
