"""W4A16 entry points with the reference's Python surface (roofline/kernels.py).

Weight format (roofline/kernels.py:1-13, 24-47), kept bit for bit:
  packed: int32 [K/8, N]; word (j, n) holds rows 8j..8j+7 of column n, nibble
          i at bits 4i..4i+3 storing q = clamp(round(w / s) + 8, 0, 15).
  scales: fp16 [K/128, N], s = fp16(max|w| / 7) per 128-row group.
  dequant: w = (q - 8) * s.

Every function here launches a kernel of libw4b200.so on the current CUDA
stream through the C ABI (include/w4b200.h). There is no CPU path: a CPU
tensor is moved to the current CUDA device first, and the call fails if the
library or a GPU is missing.
"""
from __future__ import annotations

import contextlib
import ctypes
import json
import os
import threading
from pathlib import Path

import torch

from . import _lib
from ._lib import GemvConfig, check

GROUP_SIZE = 128  # roofline/kernels.py:21

# Tuned tile per (device name, M, K, N, x dtype, split request, warps
# request) -> GemvConfig tuple. Mirrors roofline/kernels.py:160
# _TUNE_CACHE, which keyed num_warps by (K, N, split_k).
_TUNE_CACHE: dict[tuple, tuple[int, int, int, int, int]] = {}
_TUNE_LOCK = threading.Lock()
TUNED_CONFIG_PATH = Path(__file__).resolve().with_name("tuned_configs.json")
_loaded_tuned_file = False

_DTYPE_CODE = {torch.float16: _lib.W4_F16, torch.bfloat16: _lib.W4_BF16}
_PACK_DTYPE_CODE = {torch.float16: _lib.W4_PACK_F16, torch.bfloat16: _lib.W4_PACK_BF16,
                    torch.float32: _lib.W4_PACK_F32}


def _device_index(device: torch.device) -> int:
    return torch.cuda.current_device() if device.index is None else device.index


try:  # the raw handle of torch's current stream, without building a Stream object
    _raw_stream = torch._C._cuda_getCurrentRawStream
except AttributeError:  # pragma: no cover - other torch builds
    _raw_stream = None


def _stream_ptr(device: torch.device) -> int:
    if _raw_stream is not None:
        return _raw_stream(_device_index(device))
    return torch.cuda.current_stream(device).cuda_stream


def _on_device(device: torch.device):
    """torch.cuda.device(device), or nothing when it is already current."""
    if _device_index(device) == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device)


def _on_cuda(t: torch.Tensor) -> torch.Tensor:
    if t.is_cuda:
        return t
    if not torch.cuda.is_available():
        raise RuntimeError("roofline_decoding_b200 kernels need a CUDA device (sm_100a)")
    return t.to(torch.device("cuda", torch.cuda.current_device()))


def pack_weights(w_fp16: torch.Tensor, group_size: int = GROUP_SIZE):
    """Packs a float [K, N] weight into int4 words plus fp16 group scales.

    Same contract as roofline/kernels.py:24-47: returns (packed, scales) with
    packed int32 (K//8, N) and scales fp16 (K//group_size, N), on the device
    of the input. The quantisation runs in a CUDA kernel (w4_pack) and is
    bit-exact with the reference's torch ops for every group with a non-zero
    scale.
    """
    assert w_fp16.dim() == 2
    K, N = w_fp16.shape
    assert K % group_size == 0
    assert K % 8 == 0
    src_device = w_fp16.device
    w = _on_cuda(w_fp16)
    if w.dtype not in _PACK_DTYPE_CODE:
        w = w.float()
    w = w.contiguous()
    packed = torch.empty((K // 8, N), dtype=torch.int32, device=w.device)
    scales = torch.empty((K // group_size, N), dtype=torch.float16, device=w.device)
    with _on_device(w.device):
        check(_lib.load().w4_pack(w.data_ptr(), _PACK_DTYPE_CODE[w.dtype], packed.data_ptr(),
                                  scales.data_ptr(), K, N, group_size, _stream_ptr(w.device)),
              "pack_weights")
    if src_device != w.device:
        packed, scales = packed.to(src_device), scales.to(src_device)
    return packed, scales


def _check_packed(packed: torch.Tensor, scales: torch.Tensor) -> tuple[int, int]:
    if packed.dim() != 2 or packed.dtype != torch.int32:
        raise ValueError(f"packed must be int32 [K/8, N], got {packed.dtype} {tuple(packed.shape)}")
    K8, N = packed.shape
    K = K8 * 8
    if scales.dtype != torch.float16 or tuple(scales.shape) != (K // GROUP_SIZE, N) \
            or K % GROUP_SIZE:
        raise ValueError(f"scales must be fp16 [{K // GROUP_SIZE}, {N}] for packed "
                         f"{tuple(packed.shape)} (group size {GROUP_SIZE}), got "
                         f"{scales.dtype} {tuple(scales.shape)}")
    if not packed.is_cuda or scales.device != packed.device:
        raise ValueError("packed and scales must be on the same CUDA device")
    return K, N


def dequantize_v1(packed: torch.Tensor, scales: torch.Tensor,
                  out_dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """Materialises the dense [K, N] weight (roofline/kernels.py:77-90).

    out[k, n] = (q - 8) * s computed in fp32 and rounded once to out_dtype
    (fp16 as in the reference; bf16 is an extension).
    """
    K, N = _check_packed(packed, scales)
    if out_dtype not in _DTYPE_CODE:
        raise ValueError(f"out_dtype must be float16 or bfloat16, got {out_dtype}")
    packed, scales = packed.contiguous(), scales.contiguous()
    out = torch.empty((K, N), dtype=out_dtype, device=packed.device)
    with _on_device(packed.device):
        check(_lib.load().w4_dequant(packed.data_ptr(), scales.data_ptr(), out.data_ptr(),
                                     _DTYPE_CODE[out_dtype], K, N, _stream_ptr(packed.device)),
              "dequantize_v1")
    return out


def _prep_x(x: torch.Tensor, K: int, device: torch.device) -> tuple[torch.Tensor, bool]:
    squeeze = x.dim() == 1
    x2 = x.unsqueeze(0) if squeeze else x
    if x2.dim() != 2 or x2.shape[1] != K:
        raise ValueError(f"x must be [K] or [M, K] with K={K}, got {tuple(x.shape)}")
    if x2.dtype not in _DTYPE_CODE:
        raise ValueError(f"x must be float16 or bfloat16, got {x2.dtype}")
    if x2.device != device:
        raise ValueError(f"x is on {x2.device}, weights on {device}")
    if not 1 <= x2.shape[0] <= 16:
        raise ValueError(f"the fused kernel takes 1..16 rows, got {x2.shape[0]}")
    return x2.contiguous(), squeeze


def _device_key(device: torch.device) -> str:
    return torch.cuda.get_device_name(device)


def _load_tuned_file() -> None:
    global _loaded_tuned_file
    if _loaded_tuned_file:
        return
    _loaded_tuned_file = True
    path = Path(os.environ.get("W4B200_TUNED_CONFIGS", TUNED_CONFIG_PATH))
    if path.exists():
        for row in json.loads(path.read_text()).get("entries", []):
            _TUNE_CACHE.setdefault(tuple(row["key"]), tuple(row["config"]))


def save_tuned_configs(path: str | os.PathLike | None = None) -> Path:
    """Writes the tuning cache to JSON (loaded again on the next import)."""
    path = Path(path) if path is not None else TUNED_CONFIG_PATH
    entries = [{"key": list(k), "config": list(v)} for k, v in sorted(_TUNE_CACHE.items())]
    path.write_text(json.dumps({"entries": entries}, indent=1) + "\n")
    return path


def _tune_key(device, M, K, N, x_dtype, y_dtype, split_k, num_warps) -> tuple:
    # the output type only changes the final store, so it is not part of the key
    del y_dtype
    return (_device_key(device), M, K, N, str(x_dtype).replace("torch.", ""),
            int(split_k or 0), int(num_warps or 0))


def default_config(M: int, K: int, N: int, split_k: int = 0, num_warps: int = 0) -> GemvConfig:
    """The library's heuristic tile for this shape (no timing)."""
    cfg = GemvConfig()
    check(_lib.load().w4_gemv_default_config(M, K, N, int(split_k or 0), int(num_warps or 0),
                                             cfg), "w4_gemv_default_config")
    return cfg


def gemv_launch(x2: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor, y: torch.Tensor,
                cfg: GemvConfig) -> None:
    """Launches the fused kernel with an explicit config (no checks beyond the C ABI's)."""
    M, K = x2.shape
    N = packed.shape[1]
    check(_lib.load().w4_gemv_ex(x2.data_ptr(), _DTYPE_CODE[x2.dtype], packed.data_ptr(),
                                 scales.data_ptr(), y.data_ptr(), _DTYPE_CODE[y.dtype], M, K, N,
                                 cfg, _stream_ptr(x2.device)), "w4_gemv")


def tuned_config(M: int, K: int, N: int, x_dtype: torch.dtype, y_dtype: torch.dtype,
                 split_k: int | None, num_warps: int | None,
                 device: torch.device | None = None, tune: bool = True,
                 streaming: bool = True) -> GemvConfig:
    """Returns the cached tile for this problem, tuning it first if allowed.

    streaming=False asks for a tile with one column tile per CTA, which an
    epilogue (bias, residual, SwiGLU) or the gathered peer output needs; it
    is tuned and cached separately when the best tile streams.
    """
    device = device or torch.device("cuda", torch.cuda.current_device())
    _load_tuned_file()
    key = _tune_key(device, M, K, N, x_dtype, y_dtype, split_k, num_warps)
    hit = _TUNE_CACHE.get(key)
    if hit is not None and (streaming or len(hit) < 6 or not hit[5]):
        return GemvConfig.from_tuple(hit)
    if not streaming:
        key = key + ("one_tile",)
        hit = _TUNE_CACHE.get(key)
        if hit is not None:
            return GemvConfig.from_tuple(hit)
    if not tune or torch.cuda.is_current_stream_capturing():
        d = default_config(M, K, N, split_k or 0, num_warps or 0)
        if not streaming and d.columns:  # the default streams for very large N
            d = GemvConfig(4, 2, 3, 1, 0)
        return d
    from .tuner import tune_gemv  # local import: the tuner pulls in timing helpers

    with _TUNE_LOCK:
        hit = _TUNE_CACHE.get(key)
        if hit is None:
            best = tune_gemv(M, K, N, x_dtype, y_dtype, split_k, num_warps, device,
                             streaming=streaming)
            _TUNE_CACHE[key] = best.as_tuple()
            hit = _TUNE_CACHE[key]
    return GemvConfig.from_tuple(hit)


def w4_matmul(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor,
              split_k: int | None = None, num_warps: int | None = None,
              out_dtype: torch.dtype | None = None, out: torch.Tensor | None = None,
              config: GemvConfig | None = None, pdl: bool = False) -> torch.Tensor:
    """Fused y = x @ dequant(W) for x [K] or [M, K] (M <= 16).

    split_k None/0 lets the tuner choose; otherwise K is cut into exactly
    split_k slices reduced in a fixed order. out_dtype defaults to fp16 (the
    reference's output type); pass x.dtype to keep bf16 activations in bf16.
    """
    K, N = _check_packed(packed, scales)
    x2, squeeze = _prep_x(x, K, packed.device)
    M = x2.shape[0]
    y_dtype = out_dtype or torch.float16
    if y_dtype not in _DTYPE_CODE:
        raise ValueError(f"out_dtype must be float16 or bfloat16, got {y_dtype}")
    if out is None:
        y = torch.empty((M, N), dtype=y_dtype, device=packed.device)
    else:
        if out.dtype != y_dtype or out.numel() != M * N or not out.is_contiguous():
            raise ValueError("out must be a contiguous tensor of M*N elements of out_dtype")
        y = out
    packed, scales = packed.contiguous(), scales.contiguous()
    with _on_device(packed.device):
        cfg = config or tuned_config(M, K, N, x2.dtype, y_dtype, split_k, num_warps,
                                     packed.device)
        if pdl and not cfg.pdl:
            cfg = cfg.with_pdl(1)
        gemv_launch(x2, packed, scales, y, cfg)
    if out is not None:
        return out
    return y[0] if squeeze else y


class GemvPlan:
    """A prepared W4A16 GEMV launch for fixed weights, rows and dtypes (w4_gemv_plan).

    The reference's gemv_v3 looks up its tune cache, sets up arguments and
    launches on every call (roofline/kernels.py:250-268). A plan does the
    look-up and the set-up (tile, kernel instance, encoded tensor maps) once;
    a call then binds x and y and launches: the cheapest host path for a loop
    that runs the same layer many times. It keeps references to the weights.
    """

    def __init__(self, packed: torch.Tensor, scales: torch.Tensor, M: int = 1,
                 x_dtype: torch.dtype = torch.float16, out_dtype: torch.dtype = torch.float16,
                 config: GemvConfig | None = None, pdl: bool = False):
        K, N = _check_packed(packed, scales)
        if x_dtype not in _DTYPE_CODE or out_dtype not in _DTYPE_CODE:
            raise ValueError("x_dtype and out_dtype must be float16 or bfloat16")
        if not 1 <= M <= 16:
            raise ValueError(f"the fused kernel takes 1..16 rows, got {M}")
        self.packed, self.scales = packed.contiguous(), scales.contiguous()
        self.M, self.K, self.N = M, K, N
        self.x_dtype, self.out_dtype = x_dtype, out_dtype
        self.device = packed.device
        lib = _lib.load()
        handle = ctypes.c_void_p()
        with _on_device(self.device):
            cfg = config or tuned_config(M, K, N, x_dtype, out_dtype, None, None, self.device)
            if pdl and not cfg.pdl:
                cfg = cfg.with_pdl(1)
            self.config = cfg
            check(lib.w4_gemv_plan_create(self.packed.data_ptr(), self.scales.data_ptr(), M, K, N,
                                          _DTYPE_CODE[x_dtype], _DTYPE_CODE[out_dtype], cfg,
                                          ctypes.byref(handle)), "w4_gemv_plan_create")
        self._handle = handle.value
        self._launch = lib.w4_gemv_plan_launch
        self._launch_host = lib.w4_gemv_plan_launch_host
        self._destroy = lib.w4_gemv_plan_destroy

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """y = x @ dequant(W); x [M, K] (or [K] when M = 1) on the plan's device."""
        if x.dtype != self.x_dtype or x.numel() != self.M * self.K or not x.is_contiguous() \
                or x.device != self.device:
            raise ValueError(f"x must be a contiguous {self.x_dtype} tensor of {self.M}x{self.K} "
                             f"elements on {self.device}")
        if out is None:
            out = torch.empty((self.M, self.N), dtype=self.out_dtype, device=self.device)
        elif out.dtype != self.out_dtype or out.numel() != self.M * self.N \
                or not out.is_contiguous() or out.device != self.device:
            raise ValueError("out must be a contiguous tensor of M*N elements of out_dtype")
        check(self._launch(self._handle, x.data_ptr(), out.data_ptr(),
                           _stream_ptr(self.device)), "w4_gemv_plan_launch")
        return out

    def launch_ptrs(self, x_host: int | None, x: int, y: int, y_host: int | None,
                    stream: int) -> None:
        """One C call on raw addresses: copy x_host -> x (if given), the GEMV into
        y, copy y -> y_host (if given), all enqueued on `stream`. The caller keeps
        the buffers alive and sized (M*K and M*N elements)."""
        check(self._launch_host(self._handle, x_host, x, y, y_host, stream),
              "w4_gemv_plan_launch_host")

    @staticmethod
    def batch(plans: "list[GemvPlan]") -> "GemvPlanBatch":
        """The plans run back to back by one call (w4_gemv_plans_launch_host)."""
        return GemvPlanBatch(plans)

    def __del__(self):
        h = getattr(self, "_handle", None)
        if h:
            self._destroy(h)
            self._handle = None


class GemvPlanBatch:
    """Plans run in order by one C call, their inputs and outputs back to back.

    x (host and device) holds every plan's M*K inputs one after another, y
    every plan's M*N outputs; the call copies x in once, runs the GEMVs and
    copies y out once. Keeps references to the plans.
    """

    def __init__(self, plans: list[GemvPlan]):
        if not plans:
            raise ValueError("a batch needs at least one plan")
        self.plans = list(plans)
        self.x_elems = sum(p.M * p.K for p in self.plans)
        self.y_elems = sum(p.M * p.N for p in self.plans)
        self._array = (ctypes.c_void_p * len(self.plans))(*[p._handle for p in self.plans])
        self._launch = _lib.load().w4_gemv_plans_launch_host

    def launch_ptrs(self, x_host: int | None, x: int, y: int, y_host: int | None,
                    stream: int) -> None:
        """Copy x_host -> x (if given), run every plan, copy y -> y_host (if given)."""
        check(self._launch(self._array, len(self.plans), x_host, x, y, y_host, stream),
              "w4_gemv_plans_launch_host")


def fused_launch(x2: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor,
                 y: torch.Tensor, cfg: GemvConfig, prologue: int = 0,
                 norm_weight: torch.Tensor | None = None, eps: float = 1e-6,
                 epilogue: int = 0, epi_src: torch.Tensor | None = None) -> None:
    """One fused GEMV launch (w4_gemv_fused): prologue on x, epilogue on y.

    prologue: _lib.W4_PRO_RMSNORM (x <- rmsnorm(x) * norm_weight) or
    _lib.W4_PRO_SWIGLU (x is [M, 2K] gate|up, x <- silu(gate) * up);
    epilogue: _lib.W4_EPI_BIAS (y += epi_src[n]), _lib.W4_EPI_RESIDUAL
    (y <- epi_src + round(y); epi_src may be y itself) or _lib.W4_EPI_SWIGLU (the
    weight columns alternate gate and up in blocks of 16 * cfg.strips; y [M, N/2]
    <- silu(gate) * up; needs a tile without split).
    """
    M = x2.shape[0]
    K = packed.shape[0] * 8
    N = packed.shape[1]
    ops = _lib.FusedOps(int(prologue), norm_weight.data_ptr() if norm_weight is not None else None,
                        float(eps), int(epilogue),
                        epi_src.data_ptr() if epi_src is not None else None)
    check(_lib.load().w4_gemv_fused(x2.data_ptr(), _DTYPE_CODE[x2.dtype], packed.data_ptr(),
                                    scales.data_ptr(), y.data_ptr(), _DTYPE_CODE[y.dtype], M, K,
                                    N, ops, cfg, _stream_ptr(x2.device)), "w4_gemv_fused")


def gemv_v2(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor,
            out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Fused GEMV, x [K] -> y [N] fp16 (roofline/kernels.py:131-145).

    The tile and the K split are the tuner's choice; the sum is reduced in a
    fixed order, so results are reproducible run to run.
    """
    return w4_matmul(x, packed, scales, split_k=None, num_warps=None, out_dtype=out_dtype)


def gemv_v3(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor, split_k: int = 1,
            num_warps: int | None = None, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Split-K fused GEMV (roofline/kernels.py:250-268).

    K is cut into exactly split_k slices (the reference snaps them to 8-row
    boundaries and sums them with fp16 atomics; here slices are whole 128-row
    groups and the fp32 partials are summed in rank order inside a
    thread-block cluster, so there are no atomics and no zero-fill launch).
    num_warps (4 or 8) fixes the number of compute warps per CTA; None lets
    the tuner pick the tile, as the reference's _tune_num_warps did.
    """
    if split_k is not None and split_k < 1:
        raise ValueError(f"split_k must be >= 1, got {split_k}")
    if num_warps is not None and num_warps not in (4, 8):
        raise ValueError(f"num_warps must be 4 or 8, got {num_warps}")
    return w4_matmul(x, packed, scales, split_k=split_k, num_warps=num_warps,
                     out_dtype=out_dtype)


def w4_gemm(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor,
            out_dtype: torch.dtype | None = None, out: torch.Tensor | None = None,
            split_k: int | None = None) -> torch.Tensor:
    """y = x @ dequantize_v1(packed, scales) on the tensor cores for any number of rows.

    The prefill path of W4Linear: the reference dequantises to an fp16 [K, N]
    copy and runs an fp32 matmul (scripts/decode_loop.py:51-55); this kernel
    dequantises tile by tile into shared memory and accumulates in fp32 with
    tcgen05. x is [M, K] (or [K]) fp16 or bf16; N must be a multiple of 128.
    split_k: None lets the library cut K where the tiles do not fill the GPU;
    1..8 forces one launch with K in that many slices (summed in a fixed order).
    """
    K, N = _check_packed(packed, scales)
    if N % 128:
        raise ValueError(f"w4_gemm needs N % 128 == 0, got N={N}")
    x2, squeeze = _prep_x_any_rows(x, K, packed.device)
    M = x2.shape[0]
    y_dtype = out_dtype or (x2.dtype if x2.dtype in _DTYPE_CODE else torch.float16)
    if y_dtype not in _DTYPE_CODE:
        raise ValueError(f"out_dtype must be float16 or bfloat16, got {y_dtype}")
    if out is None:
        y = torch.empty((M, N), dtype=y_dtype, device=packed.device)
    else:
        if out.dtype != y_dtype or out.numel() != M * N or not out.is_contiguous():
            raise ValueError("out must be a contiguous tensor of M*N elements of out_dtype")
        y = out
    lib = _lib.load()
    with _on_device(packed.device):
        _lib.check(lib.w4_gemm_ex(x2.data_ptr(), _DTYPE_CODE[x2.dtype],
                                  packed.contiguous().data_ptr(), scales.contiguous().data_ptr(),
                                  y.data_ptr(), _DTYPE_CODE[y_dtype], M, K, N, int(split_k or 0),
                                  _stream_ptr(packed.device)), "w4_gemm")
    if out is not None:
        return out
    return y[0] if squeeze else y


def _prep_x_any_rows(x: torch.Tensor, K: int, device: torch.device) -> tuple[torch.Tensor, bool]:
    """x as a contiguous [M, K] fp16/bf16 CUDA tensor for w4_gemm (any M)."""
    squeeze = x.dim() == 1
    x2 = x.reshape(1, -1) if squeeze else x.reshape(-1, x.shape[-1])
    if x2.shape[1] != K:
        raise ValueError(f"x has {x2.shape[1]} features, packed weights expect {K}")
    if x2.dtype not in _DTYPE_CODE:
        x2 = x2.half()
    x2 = x2.to(device).contiguous()
    if x2.data_ptr() % 16:
        x2 = x2.clone()
    return x2, squeeze


def reference_gemv(x_fp16: torch.Tensor, w_fp16: torch.Tensor) -> torch.Tensor:
    """Dense fp32 reference (roofline/kernels.py:271-273)."""
    return (x_fp16.float() @ w_fp16.float()).to(torch.float16)


def device_error(device: int | None = None) -> int:
    """Reads and clears the kernels' device error word (0 = no timed-out wait)."""
    if device is None:
        device = torch.cuda.current_device()
    return _lib.device_error(device)
