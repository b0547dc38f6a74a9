"""ctypes binding of libw4b200.so, the C ABI declared in include/w4b200.h.

Loading fails loudly: there is no fallback implementation behind this module.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libw4b200.so")
HEADER_PATH = Path(__file__).resolve().parent.parent / "include" / "w4b200.h"

W4_OK, W4_ERR_INVALID_ARG, W4_ERR_ALIGNMENT, W4_ERR_UNSUPPORTED, W4_ERR_CUDA, W4_ERR_DEVICE = range(6)
W4_F16, W4_BF16 = 0, 1
# w4_pack input dtypes (the reference packer accepts any float tensor and
# works on its fp32 value).
W4_PACK_F16, W4_PACK_BF16, W4_PACK_F32 = 0, 1, 2


class W4Error(RuntimeError):
    """A CUDA-side failure reported by the library."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class GemvConfig(ctypes.Structure):
    """w4_gemv_config (include/w4b200.h), as a tuple (strips, row_groups,
    stages, split, pdl, columns); a 5-tuple leaves columns 0."""
    _fields_ = [
        ("strips", ctypes.c_int),
        ("row_groups", ctypes.c_int),
        ("stages", ctypes.c_int),
        ("split", ctypes.c_int),
        ("pdl", ctypes.c_int),
        ("columns", ctypes.c_int),
    ]

    def as_tuple(self) -> tuple[int, ...]:
        t = (self.strips, self.row_groups, self.stages, self.split, self.pdl)
        return t + (self.columns,) if self.columns else t

    @classmethod
    def from_tuple(cls, t) -> "GemvConfig":
        return cls(*[int(v) for v in t])

    def with_pdl(self, pdl: int) -> "GemvConfig":
        """A copy with programmatic dependent launch switched on (1) or off (0)."""
        c = GemvConfig.from_tuple(self.as_tuple())
        c.pdl = int(pdl)
        return c

    def __repr__(self) -> str:
        return ("GemvConfig(strips=%d, row_groups=%d, stages=%d, split=%d, pdl=%d, columns=%d)"
                % (self.as_tuple() + (0,))[:6])


W4_PRO_NONE, W4_PRO_RMSNORM, W4_PRO_SWIGLU = 0, 1, 2
W4_EPI_NONE, W4_EPI_BIAS, W4_EPI_RESIDUAL, W4_EPI_SWIGLU = 0, 1, 2, 3


class FusedOps(ctypes.Structure):
    """w4_fused_ops: prologue/epilogue fused into the GEMV (include/w4b200.h)."""
    _fields_ = [
        ("prologue", ctypes.c_int),
        ("norm_weight", ctypes.c_void_p),
        ("eps", ctypes.c_float),
        ("epilogue", ctypes.c_int),
        ("epi_src", ctypes.c_void_p),
    ]


_c_int, _c_void_p, _c_size_t = ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t

# name -> (restype, argtypes); must match include/w4b200.h
class DecodeModel(ctypes.Structure):
    """w4_decode_model: dimensions and device pointers of one decoder."""
    _fields_ = [(n, ctypes.c_int) for n in ("layers", "hidden", "intermediate", "heads",
                                            "kv_heads", "head_dim", "vocab", "max_seq")] + [
        ("eps", ctypes.c_float)] + [(n, ctypes.c_void_p) for n in (
            "qkv_packed", "qkv_scales", "o_packed", "o_scales", "gu_packed", "gu_scales",
            "down_packed", "down_scales", "qkv_bias", "in_norm", "post_norm", "final_norm",
            "embed", "cos_table", "sin_table", "k_cache", "v_cache", "prompt", "prompt_len",
            "token", "pos", "logits")]


MAX_PEERS = 8
IPC_HANDLE_BYTES = 64


class PeerOut(ctypes.Structure):
    """w4_peer_out: where a column-parallel GEMV gathers its output."""
    _fields_ = [("world", ctypes.c_int), ("rank", ctypes.c_int), ("n_full", ctypes.c_int),
                ("col_off", ctypes.c_int), ("y", (ctypes.c_void_p * MAX_PEERS) * 2),
                ("flags", ctypes.c_void_p * MAX_PEERS), ("state", ctypes.c_void_p)]


SIGNATURES = {
    "w4_version": (_c_int, []),
    "w4_status_string": (ctypes.c_char_p, [_c_int]),
    "w4_last_error": (ctypes.c_char_p, []),
    "w4_init": (_c_int, [_c_int]),
    "w4_pack": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_void_p, _c_int, _c_int, _c_int,
                         _c_void_p]),
    "w4_dequant": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_int, _c_int, _c_int, _c_void_p]),
    "w4_gemv": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_int,
                         _c_int, _c_int, _c_int, _c_int, _c_void_p]),
    "w4_gemv_ex": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_int,
                            _c_int, _c_int, ctypes.POINTER(GemvConfig), _c_void_p]),
    "w4_gemv_default_config": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int,
                                        ctypes.POINTER(GemvConfig)]),
    "w4_gemv_plan_create": (_c_int, [_c_void_p, _c_void_p, _c_int, _c_int, _c_int, _c_int, _c_int,
                                     ctypes.POINTER(GemvConfig), ctypes.POINTER(_c_void_p)]),
    "w4_gemv_plan_launch": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    "w4_gemv_plan_launch_host": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                          _c_void_p]),
    "w4_gemv_plans_launch_host": (_c_int, [ctypes.POINTER(_c_void_p), _c_int, _c_void_p,
                                           _c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    "w4_gemv_plan_destroy": (_c_int, [_c_void_p]),
    "w4_gemv_fused": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_int,
                               _c_int, _c_int, _c_int, ctypes.POINTER(FusedOps),
                               ctypes.POINTER(GemvConfig), _c_void_p]),
    "w4_decode_embed": (_c_int, [_c_void_p, _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p,
                                 _c_void_p, _c_void_p, _c_int, _c_void_p]),
    "w4_decode_attention": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                     _c_void_p, _c_void_p, _c_int, _c_int, _c_int, _c_int,
                                     _c_int, _c_void_p]),
    "w4_lm_head_workspace_bytes": (_c_size_t, []),
    "w4_lm_head_argmax": (_c_int, [_c_void_p, _c_void_p, ctypes.c_float, _c_void_p, _c_int,
                                   _c_int, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                   _c_size_t, _c_int, _c_void_p]),
    "w4_lm_head_argmax_static": (_c_int, [_c_void_p, _c_void_p, ctypes.c_float, _c_void_p,
                                          _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_int,
                                          _c_void_p]),
    "w4_decode_step_scratch_bytes": (_c_int, [ctypes.POINTER(DecodeModel),
                                              ctypes.POINTER(_c_size_t)]),
    "w4_decode_step": (_c_int, [ctypes.POINTER(DecodeModel), _c_void_p, _c_size_t, _c_void_p]),
    "w4_gemm": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_int,
                         _c_int, _c_int, _c_void_p]),
    "w4_gemm_ex": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_int,
                            _c_int, _c_int, _c_int, _c_void_p]),
    "w4_gptq_block": (_c_int, [_c_void_p, _c_void_p, _c_int, _c_void_p, _c_void_p, _c_void_p,
                               _c_void_p]),
    "w4_gemv_tune": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                              ctypes.POINTER(GemvConfig), ctypes.POINTER(ctypes.c_float)]),
    "w4_peer_flag_bytes": (_c_size_t, [_c_int]),
    "w4_gemv_allgather": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_void_p, _c_int, _c_int,
                                   _c_int, _c_int, ctypes.POINTER(GemvConfig),
                                   ctypes.POINTER(PeerOut), _c_void_p]),
    "w4_peer_alloc": (_c_int, [_c_size_t, ctypes.POINTER(_c_void_p), _c_void_p]),
    "w4_peer_free": (_c_int, [_c_void_p]),
    "w4_peer_open": (_c_int, [_c_void_p, ctypes.POINTER(_c_void_p)]),
    "w4_peer_close": (_c_int, [_c_void_p]),
    "w4_device_error": (_c_int, [_c_int, ctypes.POINTER(_c_int)]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Returns the loaded library; raises if the shared object is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(
                    f"{LIB_PATH.name} is not built; run `python -c 'import __graft_entry__ as g; "
                    f"g.build()'` (or roofline_decoding_b200/_build.py) first")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    """Raises the Python exception matching a w4_status."""
    if status == W4_OK:
        return
    lib = load()
    msg = f"{what}: {lib.w4_status_string(status).decode()}: {lib.w4_last_error().decode()}"
    if status in (W4_ERR_INVALID_ARG, W4_ERR_ALIGNMENT):
        raise ValueError(msg)
    if status == W4_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise W4Error(status, msg)


def device_error(device: int) -> int:
    """Reads and clears the kernels' device-side error word (synchronises)."""
    code = ctypes.c_int(0)
    check(load().w4_device_error(device, ctypes.byref(code)), "w4_device_error")
    return code.value
