#!/usr/bin/env python3
"""Benchmark of the W4A16 GEMV path on B200 (one JSON line on rank 0).

Workload (default, --workload sweep): the per-shape batch-1 GEMV sweep of the
Qwen2.5-1.5B decode layers and the small model's layers: K x N in
1536x1536 (q/o), 1536x8960 (gate/up), 8960x1536 (down, tall K), 1536x256
(k/v), 1024x1024, 1024x2816, each with fp16 and bf16 activations, M = 1.
W ~ N(0, 0.02) fp16 packed to int4 (group 128), x ~ N(0, 1), seeded.

One step = the 12 GEMVs once, each on its own copy of the packed weights; the
copies rotate so that every launch streams its weights from HBM (the pool is
larger than 3x the L2). Steps are CUDA graphs (one per rotation slot) with a
timing event after every kernel, replayed back to back.

  value  : algorithmic bytes of all GEMVs of all ranks / max-over-ranks time
           of the timed steps, GB/s (inputs resident in HBM).
  e2e    : the same metric through the public API (w4_matmul) with x copied
           from pinned host memory and y copied back every GEMV, timed with
           events around the steps (host synchronises once per step).
  roofline: the dominant GEMV (largest share of kernel time): algorithmic bytes
           per launch / its mean event-timed duration, against the measured
           HBM copy bandwidth in MEASURED_PEAKS.json.
  cpu_baseline: the reference's dequantise-then-matmul path restated in C
           (oracle/w4_oracle.c, OpenMP) on a bounded sample, rank 0 only.

--impl reference times that CPU restatement as the reference arm.
Multi-GPU (torchrun): every rank runs the same sweep on its own GPU (the sweep
shapes are not partitioned): replicas, weak scaling, no data-path collective.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

SWEEP_SHAPES = [(1536, 1536), (1536, 8960), (8960, 1536), (1536, 256), (1024, 1024),
                (1024, 2816)]
SWEEP_DTYPES = ["fp16", "bf16"]
METRIC = "W4A16 GEMV HBM GB/s (batch-1 per-shape sweep, fp16+bf16 activations)"
WORKLOAD = ("qwen2.5-1.5b + small-model decode GEMV sweep, M=1: 1536x1536, 1536x8960, "
            "8960x1536, 1536x256, 1024x1024, 1024x2816; fp16 and bf16 activations")
FALLBACK_HBM_GBS = 6650.0


def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def gemv_bytes(M, K, N):
    return K * N // 2 + 2 * N * (K // 128) + 2 * M * K + 2 * M * N


# ---------------------------------------------------------------- distributed

def dist_setup(n_gpus):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    import torch

    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None or not self.path:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[4:9]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[3][1:])
                          if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows),
                "sm_max_mhz": max(r[1] for r in rows),
                "power_w_max": max(r[2] for r in rows), "samples": len(rows),
                "reasons": reasons}


# ---------------------------------------------------------------- CPU baseline

def cpu_cases():
    """Seeded inputs of the sweep for the CPU restatement (built outside any timing)."""
    from oracle import c_oracle
    from oracle import w4_oracle as o

    cases = []
    for K, N in SWEEP_SHAPES:
        w = o.normal_weights(K, N, seed=K * 7 + N)
        p, s = c_oracle.pack(w)
        for dt in SWEEP_DTYPES:
            x = o.activations(1, K, seed=3, bf16=(dt == "bf16"))
            cases.append((x, p, s, dt == "bf16", np.empty((K, N), dtype=np.uint16),
                          gemv_bytes(1, K, N)))
    return cases


def cpu_sweep(cases):
    """One sweep of the reference's dequantise-then-matmul path on the host cores."""
    from oracle import c_oracle

    for x, p, s, bf, wb, _ in cases:
        c_oracle.dequant_matmul(x, p, s, x_bf16=bf, wbuf=wb)


def cpu_sweep_sample(seconds=10.0, min_sweeps=1):
    """GB/s of the CPU restatement over whole sweeps for about `seconds`."""
    from oracle import c_oracle

    cases = cpu_cases()
    cpu_sweep(cases)  # warm the OpenMP pool and the pages
    sweeps, t0 = 0, time.perf_counter()
    while sweeps < min_sweeps or time.perf_counter() - t0 < seconds:
        cpu_sweep(cases)
        sweeps += 1
    dt = time.perf_counter() - t0
    total = sweeps * sum(c[5] for c in cases)
    return total / dt / 1e9, sweeps, dt, c_oracle.max_threads()


def run_reference(args, rank, world):
    """--impl reference: the CPU restatement of the reference path, rank 0 only."""
    if rank != 0:
        return
    from oracle import c_oracle

    cases = cpu_cases()
    for _ in range(args.warmup):
        cpu_sweep(cases)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_sweep(cases)
    elapsed = time.perf_counter() - t0
    cores = c_oracle.max_threads()
    bytes_step = sum(c[5] for c in cases)
    value = bytes_step * args.steps / elapsed / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(elapsed / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "w4a16 (fp32 dequantise-then-matmul)",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
        "config": {"workload": WORKLOAD, "M": 1, "parallelism": "cpu"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cores,
                         "kind": "port",
                         "sample": f"{args.steps} full sweeps (12 GEMVs each), one per step; "
                                   "oracle/w4_oracle.c dequantise-to-fp16 then fp32 GEMV, "
                                   "OpenMP"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- our arm

def build_cases(torch, device, pool_min_bytes):
    from roofline_decoding_b200 import kernels as Kn

    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    base = []
    for K, N in SWEEP_SHAPES:
        g = torch.Generator(device="cpu").manual_seed(K * 7 + N)
        w = (torch.randn((K, N), generator=g) * 0.02).half().to(device)
        p, s = Kn.pack_weights(w)
        base.append((K, N, p, s))
        del w
    weight_bytes = sum(p.numel() * 4 + s.numel() * 2 for _, _, p, s in base)
    # each step uses 2 copies (one per activation dtype); rotate over enough
    # copies that the pool exceeds 3x L2
    slots = max(2, -(-max(3 * l2, pool_min_bytes) // (2 * weight_bytes)))
    pool = []
    for _ in range(slots):
        slot = []
        for dt in SWEEP_DTYPES:
            slot.append([(K, N, p.clone(), s.clone()) for K, N, p, s in base])
        pool.append(slot)
    xs = {}
    for K, _ in SWEEP_SHAPES:
        for dt in SWEEP_DTYPES:
            tdt = torch.float16 if dt == "fp16" else torch.bfloat16
            g = torch.Generator(device="cpu").manual_seed(K)
            xs[(K, dt)] = torch.randn((1, K), generator=g).to(tdt).to(device)
    return pool, xs, slots, weight_bytes, l2


def run_ours(args, rank, world, local):
    import torch

    from roofline_decoding_b200 import kernels as Kn
    from roofline_decoding_b200.roofline import measure_copy_bandwidth_gbs

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    peak, peak_kind = measured_peaks()
    pool, xs, slots, weight_bytes, l2 = build_cases(torch, device, 0)
    tdt = {"fp16": torch.float16, "bf16": torch.bfloat16}
    ys = {(K, N, dt): torch.empty((1, N), dtype=torch.float16, device=device)
          for K, N in SWEEP_SHAPES for dt in SWEEP_DTYPES}
    # tune (or load) the tile of every shape before any capture
    cfgs = {}
    for K, N in SWEEP_SHAPES:
        for dt in SWEEP_DTYPES:
            cfgs[(K, N, dt)] = Kn.tuned_config(1, K, N, tdt[dt], torch.float16, None, None,
                                               device)
    order = [(K, N, dt) for dt in SWEEP_DTYPES for K, N in SWEEP_SHAPES]
    n_launch = len(order)

    stream = torch.cuda.Stream(device)

    def launch_all(si, pdl, ev=None):
        for i, (K, N, dt) in enumerate(order):
            p, s = pool_lookup(pool, si, K, N, dt)
            Kn.w4_matmul(xs[(K, dt)], p, s, out=ys[(K, N, dt)], config=cfgs[(K, N, dt)],
                         pdl=pdl)
            if ev is not None:
                ev[i + 1].record(stream)

    with torch.cuda.stream(stream):
        for si in range(slots):  # warm every buffer once outside capture
            launch_all(si, pdl=False)
    stream.synchronize()

    # Region A (value): one graph per rotation slot, the 12 GEMVs chained with
    # programmatic dependent launch, replayed back to back.
    # Region B (per kernel): the same launches without PDL and with an external
    # timing event after every kernel, for per-shape times and the roofline.
    def capture(si, pdl, ev):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                if ev is not None:
                    ev[0].record(stream)
                launch_all(si, pdl, ev)
        return g

    graphs_pdl = [capture(si, True, None) for si in range(slots)]
    evs = [[torch.cuda.Event(enable_timing=True, external=True) for _ in range(n_launch + 1)]
           for _ in range(slots)]
    graphs_ev = [capture(si, False, evs[si]) for si in range(slots)]
    with torch.cuda.stream(stream):  # upload every graph before any timing
        for g in graphs_pdl + graphs_ev:
            g.replay()
    torch.cuda.synchronize()

    copy_gbs = measure_copy_bandwidth_gbs(n_bytes=1 << 30, iters=10, device=device)

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            graphs_pdl[i % slots].replay()
    torch.cuda.synchronize()

    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            start.record(stream)
            for i in range(args.steps):
                graphs_pdl[(args.warmup + i) % slots].replay()
            end.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        elapsed_ms = max_over_ranks(start.elapsed_time(end), world)

        # region B: per-kernel event times, one pass over the slots at a time
        per_kernel = [[] for _ in range(n_launch)]
        done = 0
        with torch.cuda.stream(stream):
            while done < args.steps:
                n = min(slots, args.steps - done)
                for si in range(n):
                    graphs_ev[si].replay()
                stream.synchronize()
                for si in range(n):
                    for k in range(n_launch):
                        per_kernel[k].append(evs[si][k].elapsed_time(evs[si][k + 1]))
                done += n
        torch.cuda.synchronize()
    per_kernel = [[max_over_ranks(v, world) for v in ks] for ks in per_kernel] \
        if world > 1 else per_kernel

    bytes_step = sum(gemv_bytes(1, K, N) for K, N, _ in order)
    value = world * bytes_step * args.steps / (elapsed_ms / 1e3) / 1e9

    # per-shape table and the dominant kernel
    per_shape = []
    for k, (K, N, dt) in enumerate(order):
        t_us = statistics.mean(per_kernel[k]) * 1e3
        gbs = gemv_bytes(1, K, N) / (t_us * 1e-6) / 1e9
        per_shape.append({"K": K, "N": N, "act": dt, "us": round(t_us, 2),
                          "GBps": round(gbs, 1), "frac": round(gbs / peak, 4),
                          "config": list(cfgs[(K, N, dt)].as_tuple())})
    dom = max(range(n_launch), key=lambda k: sum(per_kernel[k]))
    dK, dN, ddt = order[dom]
    dom_us = statistics.mean(per_kernel[dom]) * 1e3
    achieved = gemv_bytes(1, dK, dN) / (dom_us * 1e-6) / 1e9
    kernel_total_us = sum(statistics.mean(v) * 1e3 for v in per_kernel)

    # e2e through the public API with host buffers
    e2e = run_e2e(torch, Kn, pool, cfgs, order, args, device, world)

    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            v, sweeps, dt_s, cores = cpu_sweep_sample(seconds=args.cpu_seconds)
            cpu = {"value": round(v, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                   "sample": f"{sweeps} full sweeps (12 GEMVs) in {dt_s:.1f} s of "
                             "oracle/w4_oracle.c dequantise-to-fp16 then fp32 GEMV, OpenMP"}
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(elapsed_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "w4a16 (fp32 accumulate)",
            "data": "synthetic (seeded N(0,0.02) weights packed to int4, N(0,1) activations)",
            "config": {"workload": WORKLOAD, "M": 1, "global_batch": world,
                       "parallelism": f"replicas{world}",
                       "l2": f"rotating packed-weight pool of {slots} step copies "
                             f"({slots * 2 * weight_bytes / 2**20:.0f} MiB > 3x L2 "
                             f"{l2 / 2**20:.0f} MiB)",
                       "timing": "value: CUDA graph per rotation slot, the 12 GEMVs chained "
                                 "with programmatic dependent launch, CUDA events around the "
                                 "steps, max over ranks; per_shape/roofline: the same "
                                 "launches without PDL, an event after every kernel"},
            "gpu_launches": n_launch * args.steps,  # region A
            "roofline": {"bound": "hbm", "kernel": f"w4_gemv_kernel K={dK} N={dN} act={ddt}",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": None,
                         "bytes_per_launch": gemv_bytes(1, dK, dN),
                         "mean_launch_us": round(dom_us, 3),
                         "sum_isolated_kernel_us_per_step": round(kernel_total_us, 2),
                         "pdl_chained_us_per_step": round(elapsed_ms * 1e3 / args.steps, 2)},
            "per_shape": per_shape,
            "measured_copy_gbs": round(copy_gbs, 1),
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
    line_clocks = clocks.summary()
    if rank == 0:
        line["clocks"] = line_clocks
        print(json.dumps(line), flush=True)
    del graphs_pdl, graphs_ev


def pool_lookup(pool, si, K, N, dt):
    for k2, n2, p, s in pool[si][SWEEP_DTYPES.index(dt)]:
        if (k2, n2) == (K, N):
            return p, s
    raise KeyError((K, N, dt))


def run_e2e(torch, Kn, pool, cfgs, order, args, device, world):
    """Public-API steps: pinned x -> device, fused GEMV, y -> pinned host, per GEMV."""
    hx, hy = {}, {}
    for K, N, dt in order:
        tdt = torch.float16 if dt == "fp16" else torch.bfloat16
        hx[(K, N, dt)] = torch.randn((1, K)).to(tdt).pin_memory()
        hy[(K, N, dt)] = torch.empty((1, N), dtype=torch.float16).pin_memory()
    slots = len(pool)

    def step(i):
        for K, N, dt in order:
            p, s = pool_lookup(pool, i % slots, K, N, dt)
            xd = hx[(K, N, dt)].to(device, non_blocking=True)
            y = Kn.w4_matmul(xd, p, s, config=cfgs[(K, N, dt)])
            hy[(K, N, dt)].copy_(y, non_blocking=True)
        torch.cuda.current_stream(device).synchronize()

    for i in range(args.warmup):
        step(i)
    barrier(world)
    torch.cuda.synchronize()
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_ev.record()
    for i in range(args.steps):
        step(args.warmup + i)
    e_ev.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(s_ev.elapsed_time(e_ev), world)
    bytes_step = sum(gemv_bytes(1, K, N) for K, N, _ in order)
    h2d = sum(hx[k].numel() * hx[k].element_size() for k in hx)
    d2h = sum(hy[k].numel() * hy[k].element_size() for k in hy)
    return {"value": round(world * bytes_step * args.steps / (ms / 1e3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": round(ms / args.steps, 4),
            "path": "roofline_decoding_b200.w4_matmul (C ABI w4_gemv_ex) per GEMV, "
                    "pinned H2D x, D2H y, one host sync per step"}


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    rank, world, local = dist_setup(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        else:
            run_ours(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
