"""Explicit per-shape tuner for the fused GEMV (replaces roofline/kernels.py:211-247).

The reference timed num_warps in {4, 8} with a fresh zeroed output per trial,
because its split-K kernel accumulated with atomics (kernels.py:154-159). The
kernel here writes its output without atomics, so trials can share buffers;
what matters instead is that B200's 126 MB L2 would hold every decode-sized
weight matrix, so every timed launch is preceded by a write of twice the L2
size: the tuner ranks tiles for weights streamed from HBM, as in decode.
Tuning must run outside CUDA-graph capture (it synchronises).
"""
from __future__ import annotations

import statistics

import torch

from ._lib import GemvConfig


def _candidates(M: int, K: int, N: int, split_k: int | None, num_warps: int | None,
                sm_count: int):
    from .kernels import default_config

    groups = K // 128
    warps = [num_warps] if num_warps else [4, 8]
    splits = [split_k] if split_k else [s for s in (1, 2, 3, 4, 6, 8, 12, 16) if s <= groups]
    seen = set()
    for cw in warps:
        for strips in (1, 2, 4):
            rg = cw // strips
            if rg not in (1, 2, 4, 8):
                continue
            if strips > 1 and 32 * strips > N:
                continue
            tiles = -(-N // (32 * strips))
            for split in splits:
                ctas = tiles * split
                if not split_k and split > 1 and ctas > 6 * sm_count:
                    continue  # already plenty of CTAs without splitting further
                gps = -(-groups // split)
                n_stages = -(-gps // rg)
                # up to the whole share in flight at once (small shapes are latency
                # bound: every stage that waits for a free slot costs a DRAM trip)
                for stages in (2, 3, 4, 5, 6, 8):
                    if stages > max(2, n_stages):
                        continue
                    c = (strips, rg, stages, split, 0)
                    if c not in seen:
                        seen.add(c)
                        yield GemvConfig(*c)
    d = default_config(M, K, N, split_k or 0, num_warps or 0)
    if d.as_tuple() not in seen:
        yield d


def time_config(x2, packed, scales, y, cfg: GemvConfig, flush: torch.Tensor,
                reps: int = 9, warmup: int = 2) -> float:
    """Median device time (us) of one launch with a cold L2."""
    from .kernels import gemv_launch

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
    for _ in range(warmup):
        gemv_launch(x2, packed, scales, y, cfg)
    for i in range(reps):
        flush.sum()  # evict the weights with clean lines (a write would leave dirty
        starts[i].record()  # lines whose write-back competes with the timed reads)
        gemv_launch(x2, packed, scales, y, cfg)
        ends[i].record()
    torch.cuda.synchronize()
    return statistics.median(s.elapsed_time(e) * 1e3 for s, e in zip(starts, ends))


def flush_buffer(device: torch.device) -> torch.Tensor:
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    return torch.zeros(max(2 * l2, 64 << 20) // 4, dtype=torch.float32, device=device)


def tune_gemv(M: int, K: int, N: int, x_dtype: torch.dtype, y_dtype: torch.dtype,
              split_k: int | None, num_warps: int | None, device: torch.device,
              return_table: bool = False):
    """Times every candidate tile and returns the fastest GemvConfig."""
    with torch.cuda.device(device):
        gen = torch.Generator(device=device).manual_seed(1234)
        packed = torch.randint(-2**31, 2**31 - 1, (K // 8, N), generator=gen, dtype=torch.int32,
                               device=device)
        scales = (torch.rand((K // 128, N), generator=gen, device=device) * 0.01 + 1e-3).half()
        x2 = torch.randn((M, K), generator=gen, device=device).to(x_dtype)
        y = torch.empty((M, N), dtype=y_dtype, device=device)
        flush = flush_buffer(device)
        sms = torch.cuda.get_device_properties(device).multi_processor_count
        table = []
        for cfg in _candidates(M, K, N, split_k, num_warps, sms):
            try:
                us = time_config(x2, packed, scales, y, cfg, flush)
            except (ValueError, NotImplementedError, RuntimeError):
                continue  # tile does not fit (shared memory, cluster size)
            table.append((us, cfg.as_tuple()))
        if not table:
            raise RuntimeError(f"no GEMV tile could be launched for M={M} K={K} N={N}")
        table.sort()
        best = GemvConfig.from_tuple(table[0][1])
    return (best, table) if return_table else best


# Workload shapes tuned by `python -m roofline_decoding_b200.tuner`:
# (M, K, N) of the decode sweep, the large multi-GPU shapes (full and per-rank
# column shards) and the small-M GEMM.
WORKLOAD_SHAPES = (
    [(1, k, n) for k, n in [(1536, 1536), (1536, 8960), (8960, 1536), (1536, 256),
                            (1024, 1024), (1024, 2816), (1536, 2048), (1536, 17920)]]
    + [(1, k, n // p) for k, n in [(8192, 28672), (28672, 8192), (8192, 128256)]
       for p in (1, 2, 4, 8)]
    + [(m, 4096, 14336) for m in (1, 2, 4, 8, 16)]
)


def main(argv=None) -> None:
    import argparse
    import json

    from . import kernels

    ap = argparse.ArgumentParser(description="tune the fused GEMV tile per workload shape")
    ap.add_argument("--out", default=str(kernels.TUNED_CONFIG_PATH))
    ap.add_argument("--dtypes", default="fp16,bf16")
    ap.add_argument("--quick", action="store_true", help="decode-sweep shapes only")
    args = ap.parse_args(argv)
    dev = torch.device("cuda", torch.cuda.current_device())
    dts = {"fp16": torch.float16, "bf16": torch.bfloat16}
    shapes = WORKLOAD_SHAPES[:8] if args.quick else WORKLOAD_SHAPES
    report = []
    for M, K, N in shapes:
        for name in args.dtypes.split(","):
            xdt = dts[name]
            best, table = tune_gemv(M, K, N, xdt, xdt, None, None, dev, return_table=True)
            key = kernels._tune_key(dev, M, K, N, xdt, xdt, None, None)
            kernels._TUNE_CACHE[key] = best.as_tuple()
            d = kernels.default_config(M, K, N)
            t_default = next((us for us, c in table if c == d.as_tuple()), None)
            report.append({"M": M, "K": K, "N": N, "x": name, "best": list(best.as_tuple()),
                           "best_us": round(table[0][0], 3),
                           "default": list(d.as_tuple()),
                           "default_us": None if t_default is None else round(t_default, 3),
                           "top5": [[round(us, 2), list(c)] for us, c in table[:5]],
                           "candidates": len(table)})
            print(json.dumps(report[-1]), flush=True)
    kernels.save_tuned_configs(args.out)
    print("saved", args.out)


if __name__ == "__main__":
    main()
