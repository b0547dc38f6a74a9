"""Explicit per-shape tuner for the fused GEMV (replaces roofline/kernels.py:211-247).

The reference timed num_warps in {4, 8} with a fresh zeroed output per trial,
because its split-K kernel accumulated with atomics (kernels.py:154-159). The
kernel here writes its output without atomics, so trials can share buffers.
What matters instead: B200's 126 MB L2 would hold every decode-sized weight
matrix, and a lone microsecond launch cannot be timed with events. So each
candidate tile is timed as a CUDA graph of dependent launches, each on its own
weight copy (the copies exceed 3x L2), as the GEMVs of a decode step run.
Tuning must run outside CUDA-graph capture (it synchronises).
"""
from __future__ import annotations

import statistics

import torch

from ._lib import GemvConfig


def column_options(tiles: int, split: int, sm_count: int) -> list[int]:
    """CTA-column counts to try: one CTA per tile (0), and for large N grids
    of one or two CTAs per SM in total (columns * split), each CTA column
    streaming two or more tiles back to back; also the column counts that
    give every CTA column the same number of tiles (2..8) with 0.6 to 2 CTAs
    per SM (an uneven last tile costs a whole tile's time: on 28672x8192, 37
    columns of 1.73 tiles took 37.5 us against 24.0 for 32 columns of 2)."""
    out = [0]
    for per_sm in (1, 2):
        c = max(1, (per_sm * sm_count + split // 2) // split)
        if 2 * c <= tiles and c not in out:
            out.append(c)
    for t in range(2, 9):
        c = tiles // t
        if tiles % t == 0 and 0.6 * sm_count <= c * split <= 2 * sm_count and c not in out:
            out.append(c)
    return out


def _candidates(M: int, K: int, N: int, split_k: int | None, num_warps: int | None,
                sm_count: int, streaming: bool = True):
    from .kernels import default_config

    groups = K // 128
    # 16 compute warps: the streaming tiles (one CTA per SM, several column
    # tiles per CTA column) only
    warps = [num_warps] if num_warps else [4, 8, 16]
    splits = [split_k] if split_k else [s for s in (1, 2, 3, 4, 6, 8, 12, 16) if s <= groups]
    seen = set()
    for cw in warps:
        for strips in (1, 2, 4):
            rg = cw // strips
            if rg not in (1, 2, 4, 8) or (cw == 16 and strips == 1):
                continue
            if strips > 1 and 32 * strips > N:
                continue
            tiles = -(-N // (32 * strips))
            for split in splits:
                for columns in (column_options(tiles, split, sm_count) if streaming else [0]):
                    if cw == 16 and (not columns or columns * split > sm_count + split):
                        continue  # 16-warp tiles: one CTA per SM, several tiles each
                    ctas = (columns or tiles) * split
                    if not split_k and split > 1 and ctas > 6 * sm_count:
                        continue  # already plenty of CTAs without splitting further
                    gps = -(-groups // split)
                    n_stages = -(-gps // rg) * (-(-tiles // columns) if columns else 1)
                    # up to the whole share in flight at once (small shapes are latency
                    # bound: every stage that waits for a free slot costs a DRAM trip)
                    for stages in (2, 3, 4, 5, 6, 8):
                        if stages > max(2, n_stages):
                            continue
                        if columns and (stages not in (4, 6) or split not in (1, 2, 4, 8)):
                            continue  # a streaming ring: fewer depths to try
                        c = (strips, rg, stages, split, 0) + ((columns,) if columns else ())
                        if c not in seen:
                            seen.add(c)
                            yield GemvConfig(*c)
    d = default_config(M, K, N, split_k or 0, num_warps or 0)
    if d.as_tuple() not in seen:
        yield d


def chain_length(weight_bytes: int, l2_bytes: int) -> int:
    """Launches per timed chain: enough distinct weight copies to exceed 3x L2."""
    return int(min(256, max(8, -(-3 * l2_bytes // max(1, weight_bytes)))))


def time_config(x2, pool, y, cfg: GemvConfig, reps: int = 3) -> float:
    """Per-launch device time (us) of `cfg` in a chain of dependent launches.

    The chain is one CUDA graph of len(pool) launches, each on its own copy
    of the weights (so every launch streams from HBM) and chained with
    programmatic dependent launch, the way a decode step issues its GEMVs.
    The best of `reps` replays is taken; a single launch is never timed alone
    (event timestamps are too coarse for microsecond kernels).
    """
    from .kernels import gemv_launch

    c = cfg.with_pdl(1)
    stream = torch.cuda.Stream(x2.device)
    with torch.cuda.stream(stream):
        gemv_launch(x2, *pool[0], y, c)  # validates the config before capture
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(g, stream=stream):
            for packed, scales in pool:
                gemv_launch(x2, packed, scales, y, c)
    best = float("inf")
    with torch.cuda.stream(stream):
        g.replay()  # upload
        for _ in range(reps):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            g.replay()
            b.record(stream)
            b.synchronize()
            best = min(best, a.elapsed_time(b) * 1e3 / len(pool))
    del g
    return best


def tune_gemv(M: int, K: int, N: int, x_dtype: torch.dtype, y_dtype: torch.dtype,
              split_k: int | None, num_warps: int | None, device: torch.device,
              return_table: bool = False, streaming: bool = True):
    """Times every candidate tile (in dependent chains) and returns the fastest
    (one column tile per CTA only, when streaming is False)."""
    with torch.cuda.device(device):
        gen = torch.Generator(device=device).manual_seed(1234)
        packed = torch.randint(-2**31, 2**31 - 1, (K // 8, N), generator=gen, dtype=torch.int32,
                               device=device)
        scales = (torch.rand((K // 128, N), generator=gen, device=device) * 0.01 + 1e-3).half()
        l2 = torch.cuda.get_device_properties(device).L2_cache_size
        n = chain_length(packed.numel() * 4 + scales.numel() * 2, l2)
        pool = [(packed.clone(), scales.clone()) for _ in range(n - 1)] + [(packed, scales)]
        x2 = torch.randn((M, K), generator=gen, device=device).to(x_dtype)
        y = torch.empty((M, N), dtype=y_dtype, device=device)
        sms = torch.cuda.get_device_properties(device).multi_processor_count
        table = []
        for cfg in _candidates(M, K, N, split_k, num_warps, sms, streaming):
            try:
                us = time_config(x2, pool, y, cfg)
            except (ValueError, NotImplementedError, RuntimeError):
                continue  # tile does not fit (shared memory, cluster size)
            table.append((us, cfg.as_tuple()))
        del pool
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
    kernels._load_tuned_file()  # keep the shapes this run does not tune in the saved file
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
            if best.columns:  # the one-tile-per-CTA winner, for epilogues and peer output
                kernels._TUNE_CACHE[key + ("one_tile",)] = tune_gemv(
                    M, K, N, xdt, xdt, None, None, dev, streaming=False).as_tuple()
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
