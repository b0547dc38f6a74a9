"""CPU oracle for the W4A16 path: numpy restatement of the reference's algorithm.

TEST INFRASTRUCTURE ONLY. Nothing in the product imports this module; only
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it, as
the checker. Parity is pinned: tests/test_oracle.py checks every function
here against golden vectors produced by the reference's own pack_weights
(tests/golden/make_golden.py) and against the C restatement in w4_oracle.c.

Restated from raihan-js/roofline-decoding:
  pack_weights      src/roofline/kernels.py:24-47
  dequantize_fp16   src/roofline/kernels.py:50-74 (_dequant_kernel: fp32 product, fp16 store)
  dequantize_f32    src/roofline/kernels.py:123-124, 203-204 (v2/v3 weights, not rounded)
  gemv_reference    tests/test_kernels.py:61-63 (x.float() @ dequantize_v1(...).float())
  gemv_exact        the v2/v3 sum (kernels.py:93-128, 163-208) in float64
"""
from __future__ import annotations

import numpy as np

GROUP_SIZE = 128


def pack_weights(w: np.ndarray, group_size: int = GROUP_SIZE, nan_as: str = "cuda"):
    """(packed int32 [K/8, N], scales float16 [K/group, N]) of a float [K, N] array.

    Steps of kernels.py:34-46: amax per (group, column) clamped at 1e-8,
    s = fp16(amax / 7) with an fp32 divide, q = clamp(rint(w / s) + 8, 0, 15)
    with an fp32 divide, nibble i of word j = row 8j + i, the shifted nibbles
    summed in int64 and wrapped to int32.

    `nan_as` fixes the int32 value of q where w / s is NaN (0/0 in a group
    whose scale underflows to 0): "cuda" -> 0 (torch's cast on a CUDA device,
    what the CUDA packer stores), "cpu" -> -2**31 (torch's cast on x86).
    """
    assert w.ndim == 2
    K, N = w.shape
    assert K % group_size == 0 and K % 8 == 0
    wf = w.astype(np.float32)
    G = K // group_size
    wg = wf.reshape(G, group_size, N)
    amax = np.abs(wg).max(axis=1, keepdims=True)                 # NaN propagates
    amax = np.maximum(amax, np.float32(1e-8))                     # clamp(min=1e-8)
    scales = (amax / np.float32(7.0)).astype(np.float16)          # [G, 1, N]
    with np.errstate(divide="ignore", invalid="ignore"):
        qf = np.rint(wg / scales.astype(np.float32)) + np.float32(8.0)
    qf = np.clip(qf, 0, 15)                                        # keeps NaN
    nan = np.isnan(qf)
    q = np.where(nan, 0, qf).astype(np.int64)
    if nan.any():
        q[nan] = 0 if nan_as == "cuda" else -(2 ** 31)
    q = q.reshape(G, group_size // 8, 8, N)
    shifts = (np.arange(8, dtype=np.int64) * 4).reshape(1, 1, 8, 1)
    summed = (q << shifts).sum(axis=2)                             # int64
    packed = summed.astype(np.uint64).astype(np.uint32).view(np.int32)  # wrap to int32
    return np.ascontiguousarray(packed.reshape(K // 8, N)), np.ascontiguousarray(scales[:, 0, :])


def unpack_nibbles(packed: np.ndarray) -> np.ndarray:
    """q values [K, N] (uint8 0..15) of a packed [K/8, N] array."""
    K8, N = packed.shape
    u = packed.view(np.uint32)
    q = np.empty((K8, 8, N), dtype=np.uint8)
    for i in range(8):
        q[:, i, :] = (u >> np.uint32(4 * i)) & np.uint32(0xF)
    return q.reshape(K8 * 8, N)


def _scales_per_row(scales: np.ndarray, K: int) -> np.ndarray:
    return np.repeat(scales.astype(np.float32), K // scales.shape[0], axis=0)


def dequantize_f32(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """(q - 8) * s in fp32, not rounded (the weights v2/v3 multiply by)."""
    q = unpack_nibbles(packed)
    return (q.astype(np.float32) - np.float32(8.0)) * _scales_per_row(scales, q.shape[0])


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16, as uint16 bit patterns."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(a)
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << np.uint32(16)).view(np.float32)


def dequantize_fp16(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """v1 dequantise (kernels.py:70-74): fp32 product rounded to fp16."""
    return dequantize_f32(packed, scales).astype(np.float16)


def dequantize_bf16_bits(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """v1 dequantise with a bf16 output (uint16 bit patterns)."""
    return f32_to_bf16_bits(dequantize_f32(packed, scales))


def as_f32(x: np.ndarray, bf16_bits: bool = False) -> np.ndarray:
    return bf16_bits_to_f32(x) if bf16_bits else x.astype(np.float32)


def gemv_reference(x: np.ndarray, packed: np.ndarray, scales: np.ndarray,
                   x_is_bf16_bits: bool = False) -> np.ndarray:
    """The reference's dequantise-then-matmul: x.float() @ fp16(dequant).float()."""
    w = dequantize_fp16(packed, scales).astype(np.float32)
    return as_f32(x, x_is_bf16_bits) @ w


def gemv_exact(x: np.ndarray, packed: np.ndarray, scales: np.ndarray,
               x_is_bf16_bits: bool = False) -> np.ndarray:
    """sum_k x[m,k] (q-8) s in float64 with fp32 weights (the v2/v3 sum, exactly)."""
    w = dequantize_f32(packed, scales).astype(np.float64)
    return as_f32(x, x_is_bf16_bits).astype(np.float64) @ w


# ---------------------------------------------------------------- seeded inputs

def normal_weights(K: int, N: int, seed: int, std: float = 0.02) -> np.ndarray:
    """W fp16 ~ N(0, std), seeded with numpy's PCG64 (the workload's distribution)."""
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((K, N), dtype=np.float32) * np.float32(std)).astype(np.float16)


def absmax_weights(K: int, N: int, seed: int) -> np.ndarray:
    """W = randn / column absmax (clamped 1e-3), fp16: tests/test_kernels.py:21-26's shape."""
    rng = np.random.default_rng(seed)
    w = rng.standard_normal((K, N), dtype=np.float32)
    w = w / np.maximum(np.abs(w).max(axis=0, keepdims=True), np.float32(1e-3))
    return w.astype(np.float16)


def activations(M: int, K: int, seed: int, bf16: bool = False) -> np.ndarray:
    """x ~ N(0, 1) as fp16 (or bf16 bit patterns), seeded."""
    rng = np.random.default_rng(seed + 7919)
    x = rng.standard_normal((M, K), dtype=np.float32)
    return f32_to_bf16_bits(x) if bf16 else x.astype(np.float16)
