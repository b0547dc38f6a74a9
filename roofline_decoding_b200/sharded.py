"""Column-parallel (N-sharded) W4A16 GEMV across the GPUs of one node.

For the large decode GEMVs (8192x28672, 28672x8192 and the 8192x128256 vocab
projection) every rank holds a contiguous copy of its slice of output columns
[r*N/P, (r+1)*N/P) of `packed` and `scales`. Columns are independent in the
reference's layout (roofline/kernels.py:24-47: words and scales are per
column), so the slice is bit-identical to packing that slice alone. x is
replicated; each rank computes y_r = x @ W[:, slice_r] with the fused kernel
and an all-gather over NVLink (NCCL) assembles y [M, N] on every rank.

Two ways to assemble y:
  gather="nccl"  the local fused GEMV, then an NCCL all-gather;
  gather="peer"  one kernel (w4_gemv_allgather) whose epilogue stores the
                 slice into every rank's output buffer over NVLink and
                 exchanges completion flags: no collective launch, no extra
                 pass over y. The buffers are CUDA-IPC mappings set up once
                 by PeerGroup.

The compute function is injectable so the sharding and NCCL gather logic can
be exercised on CPU `gloo` ranks; the default is the CUDA kernel.
"""
from __future__ import annotations

import ctypes
from typing import Callable

import torch
import torch.distributed as dist
import torch.nn as nn

from . import _lib
from .kernels import _DTYPE_CODE, _prep_x, tuned_config, w4_matmul


class _DeviceArray:
    """Zero-copy view of raw device memory for torch.as_tensor."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr,
                                         "data": (ptr, False), "version": 2, "strides": None}


class PeerGroup:
    """Device buffers that every rank of a process group can store into.

    Owns the completion flags and epoch of the gathered GEMV and, per output
    name, two y buffers [M, n_full] (alternating by epoch parity) on every
    rank, each mapped into every other rank through CUDA IPC. Construction
    and `output()` are collective: every rank calls them in the same order.
    """

    def __init__(self, group=None, device: torch.device | str | None = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _lib.MAX_PEERS:
            raise ValueError(f"at most {_lib.MAX_PEERS} ranks, got {self.world}")
        dev = torch.device(device) if device is not None else torch.device("cuda")
        self.device = dev if dev.index is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.lib = _lib.load()
        self._owned: list[int] = []
        self._opened: list[int] = []
        nbytes = int(self.lib.w4_peer_flag_bytes(self.world))
        self.flag_ptrs = self._exchange(nbytes)
        self.state = self.flag_ptrs[self.rank] + 128
        self.epoch = 0  # the device epoch, tracked on the host (one step per call)
        self.outputs: dict[str, tuple[list[list[int]], list[torch.Tensor]]] = {}

    def _exchange(self, nbytes: int) -> list[int]:
        """Allocates nbytes here, maps every rank's allocation; returns rank -> pointer."""
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * _lib.IPC_HANDLE_BYTES)()
        with torch.cuda.device(self.device):
            _lib.check(self.lib.w4_peer_alloc(nbytes, ctypes.byref(ptr), handle), "w4_peer_alloc")
        self._owned.append(ptr.value)
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=self.group)
        out = []
        for q, h in enumerate(handles):
            if q == self.rank:
                out.append(ptr.value)
                continue
            hb = (ctypes.c_ubyte * _lib.IPC_HANDLE_BYTES).from_buffer_copy(h)
            peer = ctypes.c_void_p()
            with torch.cuda.device(self.device):
                _lib.check(self.lib.w4_peer_open(hb, ctypes.byref(peer)), "w4_peer_open")
            self._opened.append(peer.value)
            out.append(peer.value)
        return out

    def output(self, name: str, M: int, n_full: int, dtype: torch.dtype):
        """Registers (collectively) the two y buffers of output `name`."""
        if name not in self.outputs:
            nbytes = (M * n_full * 2 + 255) // 256 * 256
            ptrs = [self._exchange(nbytes) for _ in range(2)]
            local = [torch.as_tensor(_DeviceArray(ptrs[b][self.rank], (M, n_full), "<i2"),
                                     device=self.device).view(dtype) for b in range(2)]
            self.outputs[name] = (ptrs, local)
        return self.outputs[name]

    def peer_out(self, name: str, n_full: int, col_off: int) -> _lib.PeerOut:
        ptrs, _ = self.outputs[name]
        po = _lib.PeerOut()
        po.world, po.rank, po.n_full, po.col_off = self.world, self.rank, n_full, col_off
        for b in range(2):
            for q in range(self.world):
                po.y[b][q] = ptrs[b][q]
        for q in range(self.world):
            po.flags[q] = self.flag_ptrs[q]
        po.state = self.state
        return po

    def sync_epoch(self) -> int:
        """Reads the device epoch (after graph replays the host count is stale)."""
        v = torch.as_tensor(_DeviceArray(self.state, (1,), "<i4"), device=self.device)
        self.epoch = int(v.item()) & 0xffffffff
        return self.epoch

    def gemv(self, x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor, name: str,
             n_full: int, col_off: int, out_dtype: torch.dtype = torch.float16,
             config: _lib.GemvConfig | None = None) -> torch.Tensor:
        """y = x @ dequant(W) on this rank's columns, gathered on every rank.

        Returns this rank's whole y [M, n_full] (a view of the buffer of this
        call's parity; valid until the call after next).
        """
        x2, squeeze = _prep_x(x, packed.shape[0] * 8, packed.device)
        M, K, N = x2.shape[0], packed.shape[0] * 8, packed.shape[1]
        _, local = self.output(name, M, n_full, out_dtype)
        cfg = config or tuned_config(M, K, N, x2.dtype, out_dtype, None, None, packed.device,
                                     streaming=False)
        po = self.peer_out(name, n_full, col_off)
        stream = torch.cuda.current_stream(packed.device).cuda_stream
        _lib.check(self.lib.w4_gemv_allgather(
            x2.data_ptr(), _DTYPE_CODE[x2.dtype], packed.data_ptr(), scales.data_ptr(),
            _DTYPE_CODE[out_dtype], M, K, N, ctypes.byref(cfg), ctypes.byref(po), stream),
            "w4_gemv_allgather")
        self.epoch += 1
        y = local[self.epoch & 1]
        return y[0] if squeeze else y

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's (after a barrier)."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for ptr in self._opened:
            self.lib.w4_peer_close(ptr)
        dist.barrier(group=self.group)
        for ptr in self._owned:
            self.lib.w4_peer_free(ptr)
        self._opened, self._owned, self.outputs = [], [], {}


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
                 matmul: Callable[..., torch.Tensor] | None = None,
                 peers: PeerGroup | None = None, name: str | None = None):
        """peers: gather through w4_gemv_allgather into `peers`' buffers (output
        `name`) instead of an NCCL all-gather."""
        super().__init__()
        self.peers = peers
        self.name = name or f"linear{id(self)}"
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
        if self.peers is not None and self.bias is None:
            c0, _ = column_range(self.out_features, self.rank, self.world)
            y = self.peers.gemv(x2, self.packed, self.scales, self.name, self.out_features, c0,
                                out_dtype).clone()
            return y.reshape(*orig[:-1], self.out_features)
        y_local = self.local_forward(x2, out_dtype)
        y = gather_columns(y_local, self.world, self.group)
        return y.reshape(*orig[:-1], self.out_features)
