"""ctypes wrapper of oracle/libw4oracle.so (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it.
"""
from __future__ import annotations

import ctypes

import numpy as np

from .build import LIB, build

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        L = ctypes.CDLL(str(LIB))
        P = ctypes.c_void_p
        i = ctypes.c_int
        L.w4o_pack.argtypes = [P, i, i, i, i, P, P]
        L.w4o_dequant_fp16.argtypes = [P, P, i, i, P]
        L.w4o_dequant_matmul.argtypes = [P, i, i, P, P, i, i, P, P]
        L.w4o_gemv_exact.argtypes = [P, i, i, P, P, i, i, P]
        L.w4o_max_threads.restype = i
        L.w4o_set_threads.argtypes = [i]
        L.w4o_set_threads.restype = i
        _lib = L
    return _lib


def _p(a: np.ndarray) -> int:
    assert a.flags.c_contiguous
    return a.ctypes.data


def pack(w: np.ndarray, group_size: int = 128, nan_as: str = "cuda"):
    K, N = w.shape
    w = np.ascontiguousarray(w.astype(np.float16)).view(np.uint16)
    packed = np.empty((K // 8, N), dtype=np.int32)
    scales = np.empty((K // group_size, N), dtype=np.uint16)
    lib().w4o_pack(_p(w), K, N, group_size, int(nan_as == "cpu"), _p(packed), _p(scales))
    return packed, scales.view(np.float16)


def dequant_fp16(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    K8, N = packed.shape
    out = np.empty((K8 * 8, N), dtype=np.uint16)
    lib().w4o_dequant_fp16(_p(packed), _p(np.ascontiguousarray(scales).view(np.uint16)),
                           K8 * 8, N, _p(out))
    return out.view(np.float16)


def dequant_matmul(x: np.ndarray, packed: np.ndarray, scales: np.ndarray, x_bf16: bool = False,
                   wbuf: np.ndarray | None = None) -> np.ndarray:
    """The reference's CPU path: fp16 dequantise, then fp32 x @ W."""
    M, K = x.shape
    N = packed.shape[1]
    if wbuf is None:
        wbuf = np.empty((K, N), dtype=np.uint16)
    y = np.empty((M, N), dtype=np.float32)
    xb = np.ascontiguousarray(x).view(np.uint16)
    lib().w4o_dequant_matmul(_p(xb), int(x_bf16), M, _p(packed),
                             _p(np.ascontiguousarray(scales).view(np.uint16)), K, N, _p(wbuf),
                             _p(y))
    return y


def gemv_exact(x: np.ndarray, packed: np.ndarray, scales: np.ndarray,
               x_bf16: bool = False) -> np.ndarray:
    M, K = x.shape
    N = packed.shape[1]
    y = np.empty((M, N), dtype=np.float64)
    xb = np.ascontiguousarray(x).view(np.uint16)
    lib().w4o_gemv_exact(_p(xb), int(x_bf16), M, _p(packed),
                         _p(np.ascontiguousarray(scales).view(np.uint16)), K, N, _p(y))
    return y


def max_threads() -> int:
    return lib().w4o_max_threads()


def use_all_cores() -> int:
    """Lets the OpenMP regions use every host core the process may run on."""
    import os

    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    return lib().w4o_set_threads(int(n or 1))
