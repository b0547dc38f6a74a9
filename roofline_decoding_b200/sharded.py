"""Column-parallel (N-sharded) W4A16 GEMV across the GPUs of one node.

For the large decode GEMVs (8192x28672, 28672x8192 and the 8192x128256 vocab
projection) every rank holds a contiguous copy of its slice of output columns
[r*N/P, (r+1)*N/P) of `packed` and `scales`. Columns are independent in the
reference's layout (roofline/kernels.py:24-47: words and scales are per
column), so the slice is bit-identical to packing that slice alone. x is
replicated; each rank computes y_r = x @ W[:, slice_r] with the fused kernel
and an all-gather over NVLink (NCCL) assembles y [M, N] on every rank.

The compute function is injectable so the sharding and gather logic can be
exercised on CPU `gloo` ranks; the default is the CUDA kernel.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist
import torch.nn as nn

from .kernels import w4_matmul


def column_range(N: int, rank: int, world: int) -> tuple[int, int]:
    """[start, end) of the columns rank `rank` owns; N must split evenly."""
    if N % world:
        raise ValueError(f"N={N} does not split evenly over {world} ranks")
    per = N // world
    if per % 8:
        raise ValueError(f"per-rank width {per} must be a multiple of 8")
    return rank * per, (rank + 1) * per


def shard_columns(packed: torch.Tensor, scales: torch.Tensor, rank: int, world: int,
                  device: torch.device | str | None = None):
    """Contiguous copies of this rank's columns of packed [K/8, N] and scales [K/128, N]."""
    c0, c1 = column_range(packed.shape[1], rank, world)
    p = packed[:, c0:c1].contiguous()
    s = scales[:, c0:c1].contiguous()
    if device is not None:
        p, s = p.to(device), s.to(device)
    return p, s


def gather_columns(y_local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gather column shards y_local [M, N/P] into y [M, N] on every rank."""
    M, n_local = y_local.shape
    buf = torch.empty((world * M, n_local), dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(buf, y_local.contiguous(), group=group)
    if M == 1:
        return buf.view(1, world * n_local)  # rank blocks are already column order
    return buf.view(world, M, n_local).permute(1, 0, 2).reshape(M, world * n_local)


class ShardedW4Linear(nn.Module):
    """A W4Linear whose output columns are split over the ranks of a process group."""

    def __init__(self, packed: torch.Tensor, scales: torch.Tensor, bias: torch.Tensor | None = None,
                 group=None, device: torch.device | str | None = None,
                 matmul: Callable[..., torch.Tensor] | None = None):
        super().__init__()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.out_features = packed.shape[1]
        self.in_features = packed.shape[0] * 8
        p, s = shard_columns(packed, scales, self.rank, self.world, device)
        self.register_buffer("packed", p)
        self.register_buffer("scales", s)
        if bias is not None:
            c0, c1 = column_range(self.out_features, self.rank, self.world)
            self.register_buffer("bias", bias[c0:c1].contiguous().to(p.device))
        else:
            self.bias = None
        self._matmul = matmul or w4_matmul

    def local_forward(self, x2: torch.Tensor, out_dtype: torch.dtype) -> torch.Tensor:
        y = self._matmul(x2, self.packed, self.scales, out_dtype=out_dtype)
        if self.bias is not None:
            y = y + self.bias.to(y.dtype)
        return y

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        orig = x.shape
        x2 = x.reshape(-1, orig[-1])
        out_dtype = x.dtype if x.dtype in (torch.float16, torch.bfloat16) else torch.float16
        y_local = self.local_forward(x2, out_dtype)
        y = gather_columns(y_local, self.world, self.group)
        return y.reshape(*orig[:-1], self.out_features)
