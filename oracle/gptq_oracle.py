"""CPU oracle for calibrated (GPTQ) int4 packing. TEST INFRASTRUCTURE ONLY.

Nothing in the product imports this module; tests/ use it as the checker.

The reference lists "Calibrated (GPTQ-style) scales to close the ppl gap" as
its next step (devto_article.md:71) and ships no implementation, so this
restates the published algorithm: GPTQ, Frantar, Ashkboos, Hoefler and
Alistarh, "GPTQ: Accurate Post-Training Quantization for Generative
Pre-trained Transformers" (2022), Algorithm 1 with lazy batch updates and
grouped scales. It is written for the reference's packed format
(src/roofline/kernels.py:24-47): symmetric group-128 scales
s = fp16(max|w| / 7) taken over the group's error-compensated weights when
the group starts, q = clamp(rint(w / s) + 8, 0, 15), nibble i of word j =
row 8j + i.

Orientation: W is [K, N] (K = in-features, the rows the packer groups), the
transpose of the paper's [rows = outputs, cols = inputs]; the Hessian of the
layer's squared output error is H = X^T X over calibration rows X [n, K].

Pinning: with a diagonal Hessian the error feedback vanishes and
gptq_quantize is exactly the reference packer (w4_oracle.pack_weights, pinned
to the reference's golden hashes); tests/test_gptq.py checks that bit for
bit, plus the defining property of the method (a lower output error than
round-to-nearest on correlated activations).
"""
from __future__ import annotations

import numpy as np

from . import w4_oracle as o

BLOCK = 128  # one quantisation group per GPTQ block


def prepare_hinv(H: np.ndarray, damp: float = 0.01):
    """Upper Cholesky factor U of H^-1 (H^-1 = U^T U) after GPTQ's conditioning.

    Steps of the paper's reference procedure: inputs that never fire (zero
    diagonal) get H[i, i] = 1 and are quantised as zero weights; then
    H += damp * mean(diag(H)) * I. Returns (U float64 [K, K], dead bool [K]).
    """
    H = np.array(H, dtype=np.float64, copy=True)
    dead = np.diag(H) == 0
    H[dead, dead] = 1.0
    H[np.diag_indices_from(H)] += damp * float(np.mean(np.diag(H)))
    L = np.linalg.cholesky(H)                        # H = L L^T
    Linv = np.linalg.inv(L)
    Hinv = Linv.T @ Linv                             # H^-1
    U = np.linalg.cholesky(Hinv).T                   # H^-1 = U^T U, U upper
    return U, dead


def gptq_block(w1: np.ndarray, hinv1: np.ndarray):
    """One 128-row block (= one group) in float32, operation for operation as
    the CUDA kernel: returns (q uint8 [128, N], scale fp16 [N], err f32 [128, N]).

    Per row i, in order: q = clamp(rint(w / s) + 8, 0, 15) (NaN -> 0, as the
    CUDA packer); err = (w - (q - 8) * s) / U[i, i]; every later row j of the
    block: w[j] = w[j] - fl(U[i, j] * err) (a product rounded to fp32, then a
    rounded subtraction - no fused multiply-add).
    """
    w = np.array(w1, dtype=np.float32, copy=True)
    h = np.asarray(hinv1, dtype=np.float32)
    B, N = w.shape
    assert B == BLOCK and h.shape == (B, B)
    amax = np.abs(w).max(axis=0)
    amax = np.maximum(amax, np.float32(1e-8))
    scale = (amax / np.float32(7.0)).astype(np.float16)
    s = scale.astype(np.float32)
    q = np.zeros((B, N), dtype=np.uint8)
    err = np.zeros((B, N), dtype=np.float32)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        for i in range(B):
            qf = np.rint(w[i] / s) + np.float32(8.0)
            qf = np.clip(qf, 0, 15)
            qf = np.where(np.isnan(qf), np.float32(0.0), qf).astype(np.float32)
            q[i] = qf.astype(np.uint8)
            wq = (qf - np.float32(8.0)) * s
            e = (w[i] - wq) / h[i, i]
            err[i] = e
            if i + 1 < B:
                w[i + 1:] = w[i + 1:] - h[i, i + 1:, None] * e[None, :]
    return q, scale, err


def pack_q(q: np.ndarray) -> np.ndarray:
    """int32 [K/8, N] words of q values [K, N] (nibble i of word j = row 8j + i)."""
    K, N = q.shape
    qq = q.astype(np.uint32).reshape(K // 8, 8, N)
    words = np.zeros((K // 8, N), dtype=np.uint32)
    for i in range(8):
        words |= qq[:, i, :] << np.uint32(4 * i)
    return words.view(np.int32)


def gptq_quantize(w: np.ndarray, H: np.ndarray, damp: float = 0.01):
    """(packed int32 [K/8, N], scales fp16 [K/128, N]) of W [K, N] calibrated on H.

    Blocks of 128 rows in order; after each block the later rows take the
    lazy batch update W[b1:] -= U[b0:b1, b1:]^T @ Err (fp32).
    """
    K, N = w.shape
    assert K % BLOCK == 0
    U, dead = prepare_hinv(H, damp)
    U32 = U.astype(np.float32)
    W = np.array(w, dtype=np.float32, copy=True)
    W[dead, :] = 0.0
    qs, scales = [], []
    for b0 in range(0, K, BLOCK):
        b1 = b0 + BLOCK
        q, sc, err = gptq_block(W[b0:b1], U32[b0:b1, b0:b1])
        qs.append(q)
        scales.append(sc)
        if b1 < K:
            W[b1:] -= U32[b0:b1, b1:].T @ err
    return pack_q(np.concatenate(qs)), np.stack(scales)


def rtn_quantize(w: np.ndarray):
    """Round-to-nearest: the reference packer itself."""
    return o.pack_weights(np.asarray(w, dtype=np.float32))


def output_error(x: np.ndarray, w: np.ndarray, packed: np.ndarray, scales: np.ndarray) -> float:
    """||X W - X dequant(packed, scales)||_F^2 / ||X W||_F^2 (float64)."""
    x64 = np.asarray(x, dtype=np.float64)
    ref = x64 @ np.asarray(w, dtype=np.float64)
    got = x64 @ o.dequantize_f32(packed, scales).astype(np.float64)
    return float(np.sum((ref - got) ** 2) / np.sum(ref ** 2))


def correlated_activations(n: int, K: int, seed: int, rank: int = 32) -> np.ndarray:
    """Calibration rows with the low-rank-plus-outlier structure of LLM
    activations: a few shared directions, a few large channels, noise."""
    rng = np.random.default_rng(seed)
    basis = rng.standard_normal((rank, K)).astype(np.float32)
    coef = rng.standard_normal((n, rank)).astype(np.float32)
    x = coef @ basis / np.sqrt(rank) + 0.3 * rng.standard_normal((n, K)).astype(np.float32)
    outliers = rng.choice(K, size=max(1, K // 64), replace=False)
    x[:, outliers] *= 8.0
    return x.astype(np.float32)
