"""Roofline accounting for batch-1 decoding on B200 (roofline/roofline.py of the reference).

Batch-1 decode is HBM-bound: a token reads every weight byte once plus the
KV cache, so tokens/s <= measured bandwidth / bytes per token. The bandwidth
is measured (device copy timed with CUDA events), never quoted, and the
bytes are counted from the architecture.

Same API as roofline/roofline.py:23-157 (model dicts, parameter counts,
bytes per token, measured copy bandwidth, ceilings, % of roofline), plus the
byte accounting the kernels are measured against: gemv_bytes (one fused GEMV) and
decode_step_bytes (the W4A16 model actually run: int4 linears, bf16 lm_head).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

# Nominal HBM3e bandwidth of an HGX B200 (8 TB/s on DGX). Measured, never used
# as a denominator.
SPEC_BANDWIDTH_GBS = 7700.0

QWEN_15B = {  # roofline/roofline.py:23-32
    "name": "Qwen2.5-1.5B-Instruct",
    "hidden": 1536,
    "layers": 28,
    "heads": 12,
    "kv_heads": 2,
    "intermediate": 8960,
    "vocab": 151936,
    "tied_embeddings": True,
}

ORCH_FUSION = {  # roofline/roofline.py:34-43 (shapes only)
    "name": "ORCH-Fusion",
    "hidden": 1024,
    "layers": 24,
    "heads": 16,
    "kv_heads": 4,
    "intermediate": 2816,
    "vocab": 2103,
    "tied_embeddings": False,
}

GROUP_SIZE = 128


@dataclass
class RooflineResult:
    model: str
    dtype: str
    weight_bytes: int
    weight_gb: float
    kv_bytes_per_token: int
    measured_bandwidth_gbs: float
    ceiling_tok_s: float


def bytes_per_param(dtype: str) -> float:
    return {"bf16": 2.0, "fp16": 2.0, "int8": 1.0, "int4": 0.5}[dtype]


def count_decoder_params(cfg: dict, include_norm: bool = True) -> dict[str, int]:
    """Parameter count per component of a GQA Llama-style decoder (biases excluded)."""
    h, n_layers, inter = cfg["hidden"], cfg["layers"], cfg["intermediate"]
    kv_dim = h // cfg["heads"] * cfg["kv_heads"]
    attn = 2 * h * h + 2 * h * kv_dim          # q, o: h x h; k, v: h x kv_dim
    mlp = 3 * h * inter                        # gate, up, down
    norms = 2 * h if include_norm else 0
    decoder = n_layers * (attn + mlp + norms)
    embed = cfg["vocab"] * h
    head = 0 if cfg["tied_embeddings"] else cfg["vocab"] * h
    final_norm = h if include_norm else 0
    total = decoder + embed + head + final_norm
    return {"decoder": decoder, "embed": embed, "head": head, "final_norm": final_norm,
            "total": total, "non_embedding": decoder + final_norm}


def weight_bytes_per_token(cfg: dict, dtype: str) -> int:
    """Weight bytes read per decoded token if every parameter had `dtype`."""
    return int(count_decoder_params(cfg)["total"] * bytes_per_param(dtype))


def kv_bytes_per_token(cfg: dict, dtype: str, seq_len: int = 2048) -> int:
    """KV-cache bytes read per token at `seq_len` positions (K and V, all layers)."""
    kv_dim = cfg["hidden"] // cfg["heads"] * cfg["kv_heads"]
    return int(2 * cfg["layers"] * kv_dim * seq_len * bytes_per_param(dtype))


def measure_copy_bandwidth_gbs(n_bytes: int = 1 << 30, iters: int = 20,
                               device: str | torch.device = "cuda") -> float:
    """Device-to-device copy bandwidth in GB/s (read + write bytes), CUDA-event timed.

    Same method as roofline/roofline.py:95-111 (torch copy_ of an n_bytes
    buffer, reads and writes counted) with the host clock replaced by CUDA
    events on the copying stream; best of `iters`.
    """
    a = torch.empty(n_bytes // 4, dtype=torch.float32, device=device)
    b = torch.empty_like(a)
    for _ in range(5):
        b.copy_(a)
    torch.cuda.synchronize(device)
    best = float("inf")
    for _ in range(iters):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        b.copy_(a)
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e) / 1e3)
    return (2 * n_bytes / 1e9) / best


def decode_ceiling(cfg: dict, dtype: str, bandwidth_gbs: float,
                   seq_len: int = 2048) -> RooflineResult:
    """Batch-1 ceiling: bandwidth / (all weights in `dtype` + KV read)."""
    wb = weight_bytes_per_token(cfg, dtype)
    kvb = kv_bytes_per_token(cfg, dtype, seq_len)
    return RooflineResult(model=cfg["name"], dtype=dtype, weight_bytes=wb, weight_gb=wb / 1e9,
                          kv_bytes_per_token=kvb, measured_bandwidth_gbs=bandwidth_gbs,
                          ceiling_tok_s=bandwidth_gbs * 1e9 / (wb + kvb))


def ceilings_table(bandwidth_gbs: float, seq_len: int = 2048) -> list[dict]:
    """Ceilings for both models x {bf16, int8, int4}."""
    rows = []
    for cfg in (QWEN_15B, ORCH_FUSION):
        for dtype in ("bf16", "int8", "int4"):
            r = decode_ceiling(cfg, dtype, bandwidth_gbs, seq_len)
            rows.append({"model": r.model, "dtype": dtype, "weight_gb": round(r.weight_gb, 3),
                         "kv_mb_per_token": round(r.kv_bytes_per_token / 1e6, 2),
                         "bandwidth_gbs": round(r.measured_bandwidth_gbs, 1),
                         "ceiling_tok_s": round(r.ceiling_tok_s, 1)})
    return rows


def achieved_bandwidth_percent(measured_tok_s: float, weight_gb: float, kv_mb_per_token: float,
                               peak_bandwidth_gbs: float) -> dict:
    """Achieved GB/s and % of the peak implied by a tok/s figure."""
    bytes_per_token = weight_gb * 1e9 + kv_mb_per_token * 1e6
    achieved = measured_tok_s * bytes_per_token / 1e9
    return {"achieved_gbs": round(achieved, 1),
            "percent_of_roofline": round(100 * achieved / peak_bandwidth_gbs, 1)}


# ----------------------------------------------------------------- this build's accounting

def gemv_bytes(M: int, K: int, N: int, act_bytes: int = 2, out_bytes: int = 2) -> int:
    """Algorithmic HBM bytes of one fused W4A16 GEMV.

    Packed int4 weights (K*N/2) + fp16 scales (2*N*K/128) + activations
    (M*K) + outputs (M*N). Any split-K workspace is not counted.
    """
    return K * N // 2 + 2 * N * (K // GROUP_SIZE) + act_bytes * M * K + out_bytes * M * N


def w4_linear_bytes(K: int, N: int) -> int:
    """Weight bytes of one int4 linear: packed words + fp16 scales."""
    return K * N // 2 + 2 * N * (K // GROUP_SIZE)


def decode_step_bytes(cfg: dict = QWEN_15B, seq_len: int = 2048, lm_head_bytes: int = 2,
                      act_bytes: int = 2) -> dict[str, int]:
    """HBM bytes one batch-1 decode step reads in the W4A16 model that is run.

    Every decoder linear is int4 (packed + scales); the tied embedding /
    lm_head stays dense (`lm_head_bytes` per parameter) and is read once for
    the logits; q/k/v biases, RMSNorm weights, one embedding row and the KV
    cache over `seq_len` positions complete the step.
    """
    h, inter, n_layers = cfg["hidden"], cfg["intermediate"], cfg["layers"]
    kv_dim = h // cfg["heads"] * cfg["kv_heads"]
    shapes = [(h, h), (h, kv_dim), (h, kv_dim), (h, h), (h, inter), (h, inter), (inter, h)]
    linears = n_layers * sum(w4_linear_bytes(k, n) for k, n in shapes)
    packed = n_layers * sum(k * n // 2 for k, n in shapes)
    lm_head = cfg["vocab"] * h * lm_head_bytes
    biases = n_layers * (h + 2 * kv_dim) * act_bytes
    norms = (2 * n_layers + 1) * h * act_bytes
    embed_row = h * act_bytes
    kv = 2 * n_layers * kv_dim * act_bytes * seq_len
    total = linears + lm_head + biases + norms + embed_row + kv
    return {"w4_linears": linears, "w4_packed": packed, "w4_scales": linears - packed,
            "lm_head": lm_head, "biases": biases, "norms": norms, "embed_row": embed_row,
            "kv_read": kv, "total": total}
