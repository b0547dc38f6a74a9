"""Calibrated int4 packing (GPTQ) in the reference's packed format.

The reference quantises by round-to-nearest (src/roofline/kernels.py:24-47)
and names the next step "Calibrated (GPTQ-style) scales to close the ppl
gap" (devto_article.md:71). This module is that step: GPTQ (Frantar et al.,
2022, Algorithm 1, lazy batch updates, one scale group per 128-row block)
producing the same (packed int32 [K/8, N], scales fp16 [K/128, N]) pair, so
every kernel of the library runs the calibrated weights unchanged.

Work split: the Hessian H = X^T X of each layer's inputs is accumulated with
GEMMs; its conditioning and Cholesky factors are computed once per layer in
float64; every 128-row block is quantised by the CUDA kernel w4_gptq_block
(the sequential part: quantise a row, feed its error into the later rows of
the block); the later blocks take the block's error in one fp32 GEMM.
"""
from __future__ import annotations

from collections.abc import Iterable

import torch
import torch.nn as nn

from . import _lib
from ._lib import check
from .kernels import GROUP_SIZE, _stream_ptr

BLOCK = 128  # rows per GPTQ block: one scale group


def accumulate_hessian(x: torch.Tensor, H: torch.Tensor | None = None) -> torch.Tensor:
    """H += X^T X (fp32) for calibration inputs x [..., K]; returns H."""
    x2 = x.detach().reshape(-1, x.shape[-1]).float()
    if H is None:
        H = torch.zeros((x2.shape[1], x2.shape[1]), dtype=torch.float32, device=x2.device)
    H.addmm_(x2.T, x2)
    return H


def prepare_hinv(H: torch.Tensor, damp: float = 0.01) -> tuple[torch.Tensor, torch.Tensor]:
    """(U fp32 [K, K] upper, dead bool [K]) with H^-1 = U^T U after GPTQ's
    conditioning: inputs that never fire get H_ii = 1 (their weights are
    quantised as zeros), then H += damp * mean(diag H) * I. Float64 throughout."""
    H = H.detach().to(torch.float64).clone()
    d = torch.diagonal(H)
    dead = d == 0
    d[dead] = 1.0
    d += damp * d.mean()
    L = torch.linalg.cholesky(H)
    Hinv = torch.cholesky_inverse(L)
    U = torch.linalg.cholesky(Hinv, upper=True)
    return U.to(torch.float32), dead


def gptq_pack(w: torch.Tensor, hessian: torch.Tensor, damp: float = 0.01,
              group_size: int = GROUP_SIZE) -> tuple[torch.Tensor, torch.Tensor]:
    """Calibrated pack of w [K, N] (K = in-features) against the layer-input
    Hessian [K, K]; same output format as pack_weights.

    With a diagonal Hessian there is no error feedback and the result equals
    pack_weights(w) bit for bit.
    """
    if group_size != GROUP_SIZE:
        raise ValueError(f"group_size must be {GROUP_SIZE} (one GPTQ block per scale group)")
    if w.ndim != 2 or w.shape[0] % BLOCK != 0:
        raise ValueError(f"w must be [K, N] with K a multiple of {BLOCK}, got {tuple(w.shape)}")
    K, N = w.shape
    if tuple(hessian.shape) != (K, K):
        raise ValueError(f"hessian must be [{K}, {K}], got {tuple(hessian.shape)}")
    if not w.is_cuda:
        raise ValueError("w must be a CUDA tensor")
    dev = w.device
    lib = _lib.load()
    with torch.cuda.device(dev):
        W = w.detach().to(dtype=torch.float32).clone()
        U, dead = prepare_hinv(hessian.to(dev), damp)
        W[dead] = 0.0
        packed = torch.empty((K // 8, N), dtype=torch.int32, device=dev)
        scales = torch.empty((K // BLOCK, N), dtype=torch.float16, device=dev)
        err = torch.empty((BLOCK, N), dtype=torch.float32, device=dev)
        prec = torch.get_float32_matmul_precision()
        torch.set_float32_matmul_precision("highest")  # the feedback GEMM in full fp32
        try:
            for b0 in range(0, K, BLOCK):
                b1 = b0 + BLOCK
                u_blk = U[b0:b1, b0:b1].contiguous()
                check(lib.w4_gptq_block(W[b0:b1].data_ptr(), u_blk.data_ptr(), N,
                                        packed[b0 // 8:b1 // 8].data_ptr(),
                                        scales[b0 // BLOCK].data_ptr(), err.data_ptr(),
                                        _stream_ptr(dev)), "w4_gptq_block")
                if b1 < K:
                    W[b1:].addmm_(U[b0:b1, b1:].T, err, alpha=-1.0)
        finally:
            torch.set_float32_matmul_precision(prec)
    return packed, scales


def calibrate_linears(model: nn.Module, batches: Iterable, skip: tuple[str, ...] = (),
                      damp: float = 0.01) -> list[str]:
    """swap_linears with GPTQ: runs `batches` through the model, accumulates
    each nn.Linear's input Hessian, then replaces every Linear not matching a
    `skip` substring (scripts/decode_loop.py:61-73's walk) with a W4Linear
    packed against its Hessian. Each layer is calibrated on the full-precision
    model's activations (one pass). Batches are passed as model(b), or
    model(**b) for dicts. Returns the swapped names."""
    from .linear import W4Linear

    targets = {name: mod for name, mod in model.named_modules()
               if isinstance(mod, nn.Linear) and not any(s in name for s in skip)}
    hess: dict[str, torch.Tensor] = {}
    hooks = []
    for name, mod in targets.items():
        def hook(m, inputs, name=name):
            hess[name] = accumulate_hessian(inputs[0], hess.get(name))
        hooks.append(mod.register_forward_pre_hook(hook))
    try:
        with torch.no_grad():
            for b in batches:
                model(**b) if isinstance(b, dict) else model(b)
    finally:
        for h in hooks:
            h.remove()
    swapped = []
    for name, mod in targets.items():
        if name not in hess:
            raise RuntimeError(f"calibration batches never reached {name}")
        dev = mod.weight.device if mod.weight.is_cuda else torch.device(
            "cuda", torch.cuda.current_device())
        # the reference quantises the fp16 weight (decode_loop.py:28-32)
        w = mod.weight.detach().to(device=dev, dtype=torch.float16).T.contiguous()
        packed, scales = gptq_pack(w, hess[name].to(dev), damp=damp)
        bias = None if mod.bias is None else mod.bias.detach().to(device=dev, dtype=torch.float16)
        parent_path, _, attr = name.rpartition(".")
        parent = model.get_submodule(parent_path) if parent_path else model
        setattr(parent, attr, W4Linear.from_packed(packed, scales, bias))
        swapped.append(name)
    return swapped
