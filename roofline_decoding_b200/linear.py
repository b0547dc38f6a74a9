"""Drop-in nn.Linear replacement (scripts/decode_loop.py:23-85 of the reference).

W4Linear stores W^T packed as int4 (K = in_features, N = out_features, the
reference's layout, decode_loop.py:28-32). Forward dispatch:
  * up to 16 rows (decode, small batches): one fused W4A16 kernel launch for
    all rows (the reference ran gemv_v3 once per row for up to 8 rows,
    decode_loop.py:45-50);
  * more rows (prefill): dequantise once, then a dense matmul with fp32
    accumulation (decode_loop.py:51-55).
The output dtype follows the activation (fp16 in, fp16 out exactly as the
reference; bf16 in, bf16 out as an extension).
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .kernels import w4_gemm, dequantize_v1, pack_weights, w4_matmul

FUSED_MAX_ROWS = 16


class W4Linear(nn.Module):
    """nn.Linear with int4-packed weights; small-row calls use the fused kernel."""

    def __init__(self, linear: nn.Linear, device: torch.device | str | None = None):
        super().__init__()
        if device is None:
            device = linear.weight.device if linear.weight.is_cuda else torch.device(
                "cuda", torch.cuda.current_device())
        # Linear.weight is (out, in); store (K=in, N=out) for x @ W.
        w = linear.weight.detach().to(device=device, dtype=torch.float16).T.contiguous()
        packed, scales = pack_weights(w)
        self.register_buffer("packed", packed)
        self.register_buffer("scales", scales)
        self.in_features = linear.in_features
        self.out_features = linear.out_features
        self.has_bias = linear.bias is not None
        if self.has_bias:
            self.register_buffer("bias", linear.bias.detach().to(device=device,
                                                                  dtype=torch.float16))
        else:
            self.bias = None

    @classmethod
    def from_packed(cls, packed: torch.Tensor, scales: torch.Tensor,
                    bias: torch.Tensor | None = None) -> "W4Linear":
        """Builds a layer around already-packed weights (no quantisation)."""
        self = cls.__new__(cls)
        nn.Module.__init__(self)
        self.register_buffer("packed", packed)
        self.register_buffer("scales", scales)
        self.in_features = packed.shape[0] * 8
        self.out_features = packed.shape[1]
        self.has_bias = bias is not None
        if self.has_bias:
            self.register_buffer("bias", bias)
        else:
            self.bias = None
        return self

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        orig = x.shape
        flat = x.reshape(-1, orig[-1])
        out_dtype = x.dtype if x.dtype in (torch.float16, torch.bfloat16) else torch.float16
        if flat.dtype != out_dtype:
            flat = flat.to(out_dtype)
        if flat.shape[0] <= FUSED_MAX_ROWS:
            out = w4_matmul(flat, self.packed, self.scales, out_dtype=out_dtype)
        elif self.out_features % 128 == 0:  # prefill rows: tcgen05 GEMM, weights never in HBM
            out = w4_gemm(flat, self.packed, self.scales, out_dtype=out_dtype)
        else:
            w = dequantize_v1(self.packed, self.scales, out_dtype=out_dtype)
            out = (flat.float() @ w.float()).to(out_dtype)
        if self.bias is not None:
            out = out + self.bias.to(out_dtype)
        return out.reshape(*orig[:-1], self.out_features)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.has_bias}, int4 group=128")


def swap_linears(model: nn.Module, skip: tuple[str, ...] = ()) -> list[str]:
    """Replaces every nn.Linear with W4Linear in place; returns the swapped names.

    Same walk as scripts/decode_loop.py:61-73: names containing any `skip`
    substring are left dense.
    """
    swapped = []
    for name, mod in list(model.named_modules()):
        if not isinstance(mod, nn.Linear):
            continue
        if any(s in name for s in skip):
            continue
        parent_path, _, attr = name.rpartition(".")
        parent = model.get_submodule(parent_path) if parent_path else model
        setattr(parent, attr, W4Linear(mod))
        swapped.append(name)
    return swapped


def weight_bytes_int4(model: nn.Module) -> int:
    """Weight bytes read per token (scripts/decode_loop.py:76-85).

    int4 layers count packed words and fp16 scales; embeddings and dense
    linears count 2 bytes per parameter.
    """
    total = 0
    for mod in model.modules():
        if isinstance(mod, W4Linear):
            total += mod.packed.numel() * 4 + mod.scales.numel() * 2
        elif isinstance(mod, nn.Embedding):
            total += mod.weight.numel() * 2
        elif isinstance(mod, nn.Linear):
            total += mod.weight.numel() * 2
    return total
