#!/usr/bin/env python3
"""Benchmark of the W4A16 GEMV path on B200 (one JSON line on rank 0).

Workloads (--workload):
  sweep  (default) the per-shape batch-1 GEMV sweep of the Qwen2.5-1.5B decode
         layers and the small model's layers: K x N in 1536x1536 (q/o),
         1536x8960 (gate/up), 8960x1536 (down, tall K), 1536x256 (k/v),
         1024x1024, 1024x2816, each with fp16 and bf16 activations, M = 1.
         The default line also carries, as sub-records:
           large           the three Llama-3-70B-like GEMVs on every GPU alone
                           (per-shape us, GB/s, fraction of HBM);
           decode          batch-1 greedy decode tok/s of the Qwen2.5-1.5B
                           architecture (CUDA graph per step), its bytes-moved
                           roofline, e2e tok/s and a CPU baseline;
           column_parallel (N > 1 only) the large GEMVs split column-parallel
                           over the N GPUs with the all-gather fused into the
                           GEMV (NVLink peer stores), checked bit for bit
                           against an NCCL all-gather of each rank's slice.
         --sweep-only leaves the sub-records out.
  gemm   small-batch W4A16 GEMM, K=4096, N=14336, M in {1, 2, 4, 8, 16}.
  large  K=8192,N=28672; K=28672,N=8192; K=8192,N=128256 at M = 1; on N GPUs
         every rank holds a column slice and the output is all-gathered.
  decode batch-1 greedy decode of a random-init Qwen2.5-1.5B-architecture
         model (int4 linears, bf16 tied lm_head, static KV 2048), tok/s.
  prefill the tcgen05 W4A16 GEMM at M = 2048 rows, TFLOP/s.
W ~ N(0, 0.02) fp16 packed to int4 (group 128), x ~ N(0, 1), seeded.

GEMV workloads: one step = every GEMV of the workload once, each on its own
copy of the packed weights; copies rotate so that every launch streams its
weights from HBM (the pool exceeds 3x L2).
  value   : algorithmic bytes (K*N/2 + 2*N*K/128 + 2*M*K + 2*M*N per GEMV, the
            full unsharded GEMV) of all ranks / max-over-ranks time, GB/s.
            Region A: one CUDA graph per rotation slot with the GEMVs chained
            by programmatic dependent launch, replayed back to back.
  per_case / roofline: region B, for each GEMV a CUDA graph of PDL-chained
            launches of that GEMV alone on weight copies exceeding 3x L2
            (events around the chain, time per launch); roofline = the GEMV
            with the largest launch time, bytes per launch / that time,
            against the measured HBM copy bandwidth (MEASURED_PEAKS.json).
  e2e     : the public API (w4_matmul) with x copied from pinned host memory
            and y copied back for every GEMV, one host sync per step.
  cpu_baseline: the reference's dequantise-then-matmul path restated in C
            (oracle/w4_oracle.c, OpenMP) on a bounded sample, rank 0, N = 1.
--impl reference times that CPU restatement as the reference arm (rank 0
only; under torchrun the other ranks exit at once, without a process group).
Multi-GPU: sweep/gemm/decode run as independent replicas (weak scaling, no
data-path collective); large is column-parallel (strong scaling).
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

FALLBACK_HBM_GBS = 6650.0

WORKLOADS = {
    "sweep": {
        "cases": [(1, k, n, dt) for dt in ("fp16", "bf16")
                  for k, n in [(1536, 1536), (1536, 8960), (8960, 1536), (1536, 256),
                               (1024, 1024), (1024, 2816)]],
        "metric": "W4A16 GEMV HBM GB/s (batch-1 per-shape sweep, fp16+bf16 activations)",
        "desc": ("qwen2.5-1.5b + small-model decode GEMV sweep, M=1: 1536x1536, 1536x8960, "
                 "8960x1536, 1536x256, 1024x1024, 1024x2816; fp16 and bf16 activations"),
        "sharded": False,
    },
    "gemm": {
        "cases": [(m, 4096, 14336, "fp16") for m in (1, 2, 4, 8, 16)],
        "metric": "W4A16 small-M GEMM HBM GB/s (K=4096, N=14336, M=1,2,4,8,16)",
        "desc": "small-batch W4A16 GEMM K=4096 N=14336 at M in {1,2,4,8,16}, fp16 activations",
        "sharded": False,
    },
    "large": {
        "cases": [(1, 8192, 28672, "fp16"), (1, 28672, 8192, "fp16"), (1, 8192, 128256, "fp16")],
        "metric": "W4A16 GEMV HBM GB/s (large shapes, column-parallel over GPUs)",
        "desc": ("Llama-3-70B-like GEMVs M=1: 8192x28672, 28672x8192, vocab 8192x128256; "
                 "column-sharded with NCCL all-gather when n_gpus > 1"),
        "sharded": True,
    },
}


# dram__bytes_read.sum + dram__bytes_write.sum of one launch of w4_gemv_kernel,
# from `ncu --set full` captures (profiles/w4_gemv_kernel_*.md), keyed by
# (M, K, N of the launch); the bench reports it as roofline.traffic.
NCU_TRAFFIC = {
    (1, 1536, 8960): 7_140_096,
    (1, 8960, 1536): 7_154_944,
    # profiles/w4_gemv_kernel_stream_8192x128256_8192x28672.md: one launch each
    # of the tuned streaming tiles
    (1, 8192, 28672): 124_964_352,
    (1, 8192, 128256): 545_657_088,
}


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
        # stdout carries the one JSON line; at NCCL_DEBUG=VERSION (a default of
        # some images) NCCL prints its version line there, so that level alone
        # is dropped (debugging levels such as INFO are left as they are)
        if os.environ.get("NCCL_DEBUG", "").upper() == "VERSION":
            del os.environ["NCCL_DEBUG"]
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(values, world):
    """Element-wise max over ranks of a list of floats (one collective)."""
    if world == 1:
        return list(values)
    import torch
    import torch.distributed as dist

    t = torch.tensor(list(values), dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


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

def cpu_cases(cases):
    """Seeded inputs for the CPU restatement (built outside any timing)."""
    from oracle import c_oracle
    from oracle import w4_oracle as o

    packs = {}
    out = []
    for M, K, N, dt in cases:
        if (K, N) not in packs:
            packs[(K, N)] = c_oracle.pack(o.normal_weights(K, N, seed=K * 7 + N))
        p, s = packs[(K, N)]
        x = o.activations(M, K, seed=3, bf16=(dt == "bf16"))
        out.append((x, p, s, dt == "bf16", np.empty((K, N), dtype=np.uint16),
                    gemv_bytes(M, K, N)))
    return out


def cpu_pass(cases):
    """One pass of the reference's dequantise-then-matmul path on the host cores."""
    from oracle import c_oracle

    for x, p, s, bf, wb, _ in cases:
        c_oracle.dequant_matmul(x, p, s, x_bf16=bf, wbuf=wb)


def cpu_sample(cases_spec, seconds):
    """GB/s of the CPU restatement over whole passes for about `seconds`."""
    from oracle import c_oracle

    c_oracle.use_all_cores()
    cases = cpu_cases(cases_spec)
    cpu_pass(cases)  # warm the OpenMP pool and the pages
    passes, t0 = 0, time.perf_counter()
    while passes < 1 or time.perf_counter() - t0 < seconds:
        cpu_pass(cases)
        passes += 1
    dt = time.perf_counter() - t0
    return passes * sum(c[5] for c in cases) / dt / 1e9, passes, dt, c_oracle.max_threads()


def workload_config(wl):
    """The `config` both arms print: the workload itself, nothing about how it runs."""
    return {"workload": wl["desc"], "batch_rows": sorted({c[0] for c in wl["cases"]}),
            "gemvs_per_step": len(wl["cases"])}


def run_reference(args, rank, world):
    """--impl reference: the CPU restatement of the reference path, rank 0 only.

    No process group is made: ranks other than 0 return at once, so that
    nothing else spins on the host cores while rank 0 uses all of them.
    """
    if rank != 0:
        return
    from oracle import c_oracle

    c_oracle.use_all_cores()  # torchrun sets OMP_NUM_THREADS=1 for every rank
    wl = WORKLOADS["sweep" if args.workload in ("decode", "prefill") else args.workload]
    cases = cpu_cases(wl["cases"])
    for _ in range(args.warmup):
        cpu_pass(cases)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_pass(cases)
    elapsed = time.perf_counter() - t0
    cores = c_oracle.max_threads()
    value = sum(c[5] for c in cases) * args.steps / elapsed / 1e9
    line = {
        "impl": "reference", "metric": wl["metric"], "value": round(value, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(elapsed / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "w4a16 (fp32 dequantise-then-matmul)",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
        "config": workload_config(wl),
        "parallelism": "cpu (rank 0 only)",
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cores,
                         "kind": "port",
                         "sample": f"{args.steps} passes over the {len(cases)} GEMVs, one per "
                                   "step; oracle/w4_oracle.c dequantise-to-fp16 then fp32 "
                                   "GEMV, OpenMP"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GEMV workloads

def build_pool(torch, Kn, cases, device, rank, world, sharded):
    """Packed weights per case, rotated over enough copies to exceed 3x L2."""
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    base = {}
    for M, K, N, dt in cases:
        if (K, N) in base:
            continue
        n_loc = N // world if sharded else N
        g = torch.Generator(device=device).manual_seed(K * 7 + N + 1000 * rank)
        w = (torch.randn((K, n_loc), generator=g, device=device) * 0.02).half()
        base[(K, N)] = Kn.pack_weights(w)
        del w
    step_bytes = sum(p.numel() * 4 + s.numel() * 2 for M, K, N, dt in cases
                     for p, s in [base[(K, N)]])
    slots = max(2, -(-3 * l2 // step_bytes))
    pool = []
    for si in range(slots):
        slot = []
        for M, K, N, dt in cases:
            p, s = base[(K, N)]
            slot.append((p.clone(), s.clone()) if si else (p, s))
        pool.append(slot)
    return pool, slots, step_bytes, l2


def run_gemv_workload(args, rank, world, local, workload=None, shard=None, cpu=True):
    """Times one GEMV workload; returns its record on rank 0 (None elsewhere).

    workload defaults to --workload; shard (default: the workload's own
    setting) splits its GEMVs column-parallel over the ranks; cpu adds the
    CPU baseline on rank 0 at N = 1.
    """
    import torch

    from roofline_decoding_b200 import kernels as Kn
    from roofline_decoding_b200.roofline import measure_copy_bandwidth_gbs

    wl = WORKLOADS[workload or args.workload]
    cases = wl["cases"]
    sharded = (wl["sharded"] if shard is None else shard) and world > 1
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    peak, peak_kind = measured_peaks()
    tdt = {"fp16": torch.float16, "bf16": torch.bfloat16}
    pool, slots, step_bytes, l2 = build_pool(torch, Kn, cases, device, rank, world, sharded)
    n_loc = [N // world if sharded else N for M, K, N, dt in cases]
    xs = []
    for M, K, N, dt in cases:
        g = torch.Generator(device="cpu").manual_seed(K + M)
        xs.append(torch.randn((M, K), generator=g).to(tdt[dt]).to(device))
    ys = [torch.empty((M, n), dtype=torch.float16, device=device)
          for (M, K, N, dt), n in zip(cases, n_loc)]
    gathered = [torch.empty((world * M, n), dtype=torch.float16, device=device)
                for (M, K, N, dt), n in zip(cases, n_loc)] if sharded else None
    # the fused peer gather stores from the epilogue of one column tile per CTA
    one_tile = sharded and args.gather == "peer"
    cfgs = [Kn.tuned_config(M, K, n, tdt[dt], torch.float16, None, None, device,
                            streaming=not one_tile)
            for (M, K, N, dt), n in zip(cases, n_loc)]
    n_launch = len(cases)
    stream = torch.cuda.Stream(device)
    peers = None
    if sharded and args.gather == "peer":
        from roofline_decoding_b200.sharded import PeerGroup

        peers = PeerGroup(device=device)
        for i, (M, K, N, dt) in enumerate(cases):
            peers.output(f"case{i}", M, N, torch.float16)

    def launch_all(si, pdl, ev=None, gather=True):
        if peers is not None and gather:  # one kernel per GEMV: compute + NVLink gather
            for i, (M, K, N, dt) in enumerate(cases):
                p, s = pool[si][i]
                c = cfgs[i]
                c = c.with_pdl(1 if pdl else 0)
                peers.gemv(xs[i], p, s, f"case{i}", N, rank * n_loc[i], config=c)
            return
        for i in range(n_launch):
            p, s = pool[si][i]
            Kn.w4_matmul(xs[i], p, s, out=ys[i], config=cfgs[i], pdl=pdl)
            if ev is not None:
                ev[i + 1].record(stream)
        if sharded and gather:
            import torch.distributed as dist

            for i in range(n_launch):
                dist.all_gather_into_tensor(gathered[i], ys[i])

    with torch.cuda.stream(stream):
        for si in range(slots):  # warm every buffer once outside capture
            launch_all(si, pdl=False)
    stream.synchronize()

    gather_check = None
    if peers is not None:
        # the fused gather against an NCCL all-gather of every rank's own
        # slice, computed by the plain GEMV with the same tile: bit for bit
        import torch.distributed as dist

        ok = True
        for i, (M, K, N, dt) in enumerate(cases):
            p, s = pool[0][i]
            y_peer = peers.gemv(xs[i], p, s, f"case{i}", N, rank * n_loc[i],
                                config=cfgs[i]).clone()
            y_loc = Kn.w4_matmul(xs[i], p, s, config=cfgs[i])
            buf = torch.empty((world * M, n_loc[i]), dtype=y_loc.dtype, device=device)
            dist.all_gather_into_tensor(buf, y_loc.contiguous())
            want = buf.view(world, M, n_loc[i]).permute(1, 0, 2).reshape(M, N)
            ok &= bool(torch.equal(y_peer, want))
        torch.cuda.synchronize()
        err = Kn.device_error(local)
        flags = max_over_ranks([0.0 if ok else 1.0, float(err != 0)], world)
        gather_check = {"bit_exact": flags[0] == 0.0, "device_error": flags[1] != 0.0,
                        "against": "NCCL all-gather of each rank's w4_matmul of its slice "
                                   "(same tile), every GEMV of the workload"}

    def capture(si, pdl, ev, gather=True):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                if ev is not None:
                    ev[0].record(stream)
                launch_all(si, pdl, ev, gather)
        return g

    graphs_pdl = [capture(si, True, None) for si in range(slots)]
    graphs_gemv = [capture(si, True, None, gather=False) for si in range(slots)] \
        if sharded else []
    with torch.cuda.stream(stream):  # upload every graph before any timing
        for g in graphs_pdl + graphs_gemv:
            g.replay()
    torch.cuda.synchronize()

    copy_gbs = measure_copy_bandwidth_gbs(n_bytes=1 << 30, iters=10, device=device)

    def timed(graphs, steps, offset):
        s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(world)
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            s_ev.record(stream)
            for i in range(steps):
                graphs[(offset + i) % slots].replay()
            e_ev.record(stream)
        torch.cuda.synchronize()
        return s_ev.elapsed_time(e_ev)

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            graphs_pdl[i % slots].replay()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        ms_a = timed(graphs_pdl, args.steps, args.warmup)
        ms_gemv = timed(graphs_gemv, args.steps, args.warmup) if sharded else 0.0
        # region B: per GEMV, a chain of dependent launches of that GEMV alone
        per_kernel = [chain_time(torch, Kn, xs[k], ys[k], pool[0][k], cfgs[k], l2, stream)
                      for k in range(n_launch)]
    elapsed_ms, ms_gemv = max_over_ranks([ms_a, ms_gemv], world)
    mean_k = max_over_ranks(per_kernel, world)  # ms per launch

    full_bytes = [gemv_bytes(M, K, N) for M, K, N, dt in cases]
    local_bytes = [gemv_bytes(M, K, n) for (M, K, N, dt), n in zip(cases, n_loc)]
    bytes_step = sum(full_bytes) if sharded else sum(full_bytes) * world
    value = bytes_step * args.steps / (elapsed_ms / 1e3) / 1e9

    per_case = []
    for k, (M, K, N, dt) in enumerate(cases):
        t_us = mean_k[k] * 1e3
        gbs = local_bytes[k] / (t_us * 1e-6) / 1e9
        per_case.append({"M": M, "K": K, "N": N, "N_local": n_loc[k], "act": dt,
                         "us": round(t_us, 2), "GBps": round(gbs, 1),
                         "frac": round(gbs / peak, 4), "config": list(cfgs[k].as_tuple())})
    dom = max(range(n_launch), key=lambda k: mean_k[k])
    dM, dK, dN, ddt = cases[dom]
    dom_us = mean_k[dom] * 1e3
    achieved = local_bytes[dom] / (dom_us * 1e-6) / 1e9

    if peers is not None:
        peers.sync_epoch()  # graph replays advanced the device epoch
    e2e = run_e2e(torch, Kn, pool, cfgs, cases, xs, args, device, world, sharded, gathered,
                  n_loc, peers)
    clk = clocks.summary()
    line = None
    if rank == 0:
        cpu_rec = None
        if world == 1 and cpu and not args.no_cpu_baseline:
            v, passes, dt_s, cores = cpu_sample(cases, args.cpu_seconds)
            cpu_rec = {"value": round(v, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                       "sample": f"{passes} passes over the {len(cases)} GEMVs in {dt_s:.1f} s "
                                 "of oracle/w4_oracle.c dequantise-to-fp16 then fp32 GEMV, "
                                 "OpenMP"}
        line = {
            "metric": wl["metric"], "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(elapsed_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "strong" if sharded else "weak", "vs_baseline": None,
            "dtype": "w4a16 (fp32 accumulate)",
            "data": "synthetic (seeded N(0,0.02) weights packed to int4, N(0,1) activations)",
            "config": workload_config(wl),
            "parallelism": ((f"column-parallel{world} + all-gather fused into the GEMV "
                             "epilogue (NVLink peer stores)" if peers is not None
                             else f"column-parallel{world} + NCCL all-gather")
                            if sharded else f"replicas{world}"),
            "l2": (f"rotating packed-weight pool of {slots} step copies "
                   f"({slots * step_bytes / 2**20:.0f} MiB >= 3x L2 {l2 / 2**20:.0f} MiB)"),
            "timing": "value: CUDA graph per rotation slot, GEMVs chained with programmatic "
                      "dependent launch, events around the steps, max over ranks; "
                      "per_case/roofline: per GEMV, a CUDA graph of PDL-chained launches of "
                      "that GEMV alone, each on its own weight copy (copies exceed 3x L2), "
                      "events around the chain",
            "gpu_launches": n_launch * args.steps,
            "roofline": {"bound": "hbm",
                         "kernel": f"w4_gemv_kernel M={dM} K={dK} N={n_loc[dom]} act={ddt}",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": NCU_TRAFFIC.get((dM, dK, n_loc[dom])),
                         "bytes_per_launch": local_bytes[dom],
                         "mean_launch_us": round(dom_us, 3),
                         "timing": "mean launch of a PDL chain of this GEMV over "
                                   "weight copies exceeding 3x L2 (region B)",
                         "sum_chained_kernel_us_per_step": round(sum(mean_k) * 1e3, 2),
                         "pdl_chained_us_per_step": round(elapsed_ms * 1e3 / args.steps, 2)},
            "per_case": per_case,
            "measured_copy_gbs": round(copy_gbs, 1),
            "e2e": e2e,
            "cpu_baseline": cpu_rec,
            "clocks": clk,
        }
        if sharded:
            line["gemv_only_ms_per_step"] = round(ms_gemv / args.steps, 4)
            line["gather_ms_per_step"] = round((elapsed_ms - ms_gemv) / args.steps, 4)
            line["gather_check"] = gather_check
    del graphs_pdl, graphs_gemv  # graphs holding NCCL calls go first
    if peers is not None:
        peers.close()
    del pool
    torch.cuda.empty_cache()
    return line


def chain_time(torch, Kn, x, y, weights, cfg, l2, stream, reps=5):
    """ms per launch of one GEMV in a graph of dependent (PDL) launches.

    Every launch reads its own copy of the packed weights and the copies
    exceed 3x L2, so each launch streams from HBM as in a decode step; the
    chain is long enough that event resolution does not matter.
    """
    packed, scales = weights
    wbytes = packed.numel() * 4 + scales.numel() * 2
    n = int(min(2048, max(8, -(-3 * l2 // wbytes))))
    copies = [(packed.clone(), scales.clone()) for _ in range(n)]
    c = cfg.with_pdl(1)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(g, stream=stream):
            for pk, sc in copies:
                Kn.w4_matmul(x, pk, sc, out=y, config=c)
        g.replay()  # upload
        best = float("inf")
        for _ in range(reps):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            g.replay()
            b.record(stream)
            b.synchronize()
            best = min(best, a.elapsed_time(b) / n)
    del g, copies
    return best


def run_e2e(torch, Kn, pool, cfgs, cases, xs, args, device, world, sharded, gathered, n_loc,
            peers=None):
    """Public-API steps: pinned x -> device, fused GEMV(s), y -> pinned host.

    Unsharded GEMVs go through a batch of launch plans (kernels.GemvPlan.batch,
    C ABI w4_gemv_plans_launch_host): one C call per step enqueues one copy of
    all inputs, the GEMVs and one copy of all outputs; one host sync per step.
    """
    hx = [x.cpu().pin_memory() for x in xs]
    hy = [torch.empty((M * world if sharded else M, n), dtype=torch.float16).pin_memory()
          for (M, K, N, dt), n in zip(cases, n_loc)]
    slots = len(pool)
    # device buffers reused every step, as a serving loop would hold them
    xd_buf = [torch.empty_like(x) for x in xs]
    yd_buf = [torch.empty((M, n), dtype=torch.float16, device=device)
              for (M, K, N, dt), n in zip(cases, n_loc)]
    batches = None
    if not sharded:
        # one launch-plan batch per rotation slot: the step's inputs lie back to
        # back in one pinned buffer, its outputs in another
        batches = [Kn.GemvPlan.batch([Kn.GemvPlan(p, s, M, xs[k].dtype, torch.float16,
                                                  config=cfgs[k], pdl=True)
                                      for k, ((p, s), (M, K, N, dt))
                                      in enumerate(zip(pool[si], cases))])
                   for si in range(slots)]
        hx_all = torch.cat([x.view(torch.int16).reshape(-1) for x in hx]).pin_memory()
        hy_all = torch.empty((batches[0].y_elems,), dtype=torch.float16).pin_memory()
        xd_all = torch.empty_like(hx_all, device=device)
        yd_all = torch.empty_like(hy_all, device=device)
        ptrs = (hx_all.data_ptr(), xd_all.data_ptr(), yd_all.data_ptr(), hy_all.data_ptr())

    def step(i):
        if batches is not None:
            batches[i % slots].launch_ptrs(*ptrs, Kn._stream_ptr(device))
            torch.cuda.current_stream(device).synchronize()
            return
        for k in range(len(cases)):
            p, s = pool[i % slots][k]
            xd = xd_buf[k]
            xd.copy_(hx[k], non_blocking=True)
            if peers is not None:
                M, K, N, dt = cases[k]
                y = peers.gemv(xd, p, s, f"case{k}", N, peers.rank * n_loc[k], config=cfgs[k])
                hy[k].view(-1).copy_(y.reshape(-1), non_blocking=True)
                continue
            y = Kn.w4_matmul(xd, p, s, config=cfgs[k], out=yd_buf[k])
            if sharded:
                import torch.distributed as dist

                dist.all_gather_into_tensor(gathered[k], y)
                y = gathered[k]
            hy[k].copy_(y, non_blocking=True)
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
    ms = max_over_ranks([s_ev.elapsed_time(e_ev)], world)[0]
    full = sum(gemv_bytes(M, K, N) for M, K, N, dt in cases)
    bytes_step = full if sharded else full * world
    if batches is not None:
        path = ("roofline_decoding_b200.GemvPlan.batch(...).launch_ptrs (C ABI "
                "w4_gemv_plans_launch_host): one call per step copies the 12 inputs from pinned "
                "host memory, runs the 12 GEMVs (programmatic dependent launch) and copies the "
                "12 outputs back; reused device buffers; one host sync per step")
    else:
        path = ("roofline_decoding_b200 column-parallel GEMV per case with its all-gather, pinned "
                "H2D x, D2H y, one host sync per step")
    return {"value": round(bytes_step * args.steps / (ms / 1e3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": sum(x.numel() * x.element_size() for x in hx),
            "d2h_bytes_per_step": sum(y.numel() * y.element_size() for y in hy),
            "ms_per_step": round(ms / args.steps, 4), "path": path}


# ---------------------------------------------------------------- decode workload

PREFILL_CASES = [(2048, 4096, 14336), (2048, 1536, 8960), (2048, 8960, 1536)]


def run_prefill(args, rank, world, local):
    """tcgen05 W4A16 GEMM for prefill rows (W4Linear above 16 rows), TFLOP/s."""
    import torch

    from roofline_decoding_b200 import kernels as Kn

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    peaks = json.loads((REPO / "MEASURED_PEAKS.json").read_text()) \
        if (REPO / "MEASURED_PEAKS.json").exists() else {}
    peak = float(peaks.get("bf16_tflops", 1590.0))
    peak_kind = "measured" if peaks else "fallback"
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    one = []
    for i, (M, K, N) in enumerate(PREFILL_CASES):
        g = torch.Generator(device=device).manual_seed(100 + i + 1000 * rank)
        w = (torch.randn((K, N), generator=g, device=device) * 0.02).half()
        packed, scales = Kn.pack_weights(w)
        del w
        x = torch.randn((M, K), generator=g, device=device).half()
        one.append((x, packed, scales))
    step_bytes = sum(x.numel() * 2 + p.numel() * 4 + s.numel() * 2 + M * N * 2
                     for (x, p, s), (M, K, N) in zip(one, PREFILL_CASES))
    slots = max(2, -(-3 * l2 // step_bytes))  # every launch reads cold operands
    pool = [one] + [[(x.clone(), p.clone(), s.clone()) for x, p, s in one]
                    for _ in range(slots - 1)]
    ys = [torch.empty((M, N), dtype=torch.float16, device=device) for M, K, N in PREFILL_CASES]
    stream = torch.cuda.Stream(device)
    flops = [2.0 * M * K * N for M, K, N in PREFILL_CASES]

    def launch(si):
        for i, (x, p, s) in enumerate(pool[si]):
            Kn.w4_gemm(x, p, s, out=ys[i])

    with torch.cuda.stream(stream):
        for si in range(slots):
            launch(si)
    stream.synchronize()
    graphs = []
    for si in range(slots):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                launch(si)
        graphs.append(g)
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            graphs[i % slots].replay()
    barrier(world)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            a.record(stream)
            for i in range(args.steps):
                graphs[(args.warmup + i) % slots].replay()
            b.record(stream)
        torch.cuda.synchronize()
        ms = max_over_ranks([a.elapsed_time(b)], world)[0]
        # per case: graphs of that GEMM alone over the rotation
        per = []
        for i in range(len(PREFILL_CASES)):
            gs = []
            for si in range(slots):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.stream(stream):
                    with torch.cuda.graph(g, stream=stream):
                        for _ in range(4):
                            x, p, s = pool[si][i]
                            Kn.w4_gemm(x, p, s, out=ys[i])
                gs.append(g)
            with torch.cuda.stream(stream):
                for g in gs:
                    g.replay()
                c, d = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                c.record(stream)
                for r in range(20):
                    gs[r % slots].replay()
                d.record(stream)
            d.synchronize()
            per.append(c.elapsed_time(d) / 80)
            del gs
    per = max_over_ranks(per, world)
    # dense comparisons on the same shapes: the reference's path (fp16 copy of
    # the weights by dequantize_v1, then an fp32 matmul) and fp16 cuBLAS on
    # that copy
    ref_ms, cublas_ms = [], []
    for (x, p, s), (M, K, N) in zip(one, PREFILL_CASES):
        for kind in ("ref", "cublas"):
            def f():
                wd = Kn.dequantize_v1(p, s)
                return (x.float() @ wd.float()).half() if kind == "ref" else x @ wd
            for _ in range(2):
                f()
            torch.cuda.synchronize()
            c, d = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            c.record()
            for _ in range(5):
                f()
            d.record()
            d.synchronize()
            (ref_ms if kind == "ref" else cublas_ms).append(c.elapsed_time(d) / 5)
    # e2e: x from pinned host memory, y back to pinned host memory, per GEMM
    hx = [x.cpu().pin_memory() for x, _, _ in one]
    hy = [torch.empty((M, N), dtype=torch.float16).pin_memory() for M, K, N in PREFILL_CASES]
    e_steps = max(3, args.steps // 10)
    torch.cuda.synchronize()
    c, d = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c.record()
    for _ in range(e_steps):
        for i, (x, p, s) in enumerate(one):
            y = Kn.w4_gemm(hx[i].to(device, non_blocking=True), p, s)
            hy[i].copy_(y, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    d.record()
    torch.cuda.synchronize()
    e_ms = max_over_ranks([c.elapsed_time(d)], world)[0]
    clk = clocks.summary()
    if rank != 0:
        return None
    dom = max(range(len(per)), key=lambda i: per[i])
    tot_flops = sum(flops)
    line = {
        "metric": "W4A16 prefill GEMM TFLOP/s (tcgen05, M=2048 tokens)",
        "value": round(tot_flops * world * args.steps / (ms / 1e3) / 1e12, 2),
        "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16 x fp16 (dequantised int4), fp32 accumulate",
        "data": "synthetic (seeded N(0,0.02) weights packed to int4, N(0,1) activations)",
        "config": {"workload": "W4A16 GEMM M=2048: 2048x4096x14336, 2048x1536x8960, 2048x8960x1536",
                   "parallelism": f"replicas{world}",
                   "l2": f"rotating operand pool of {slots} copies ({slots * step_bytes / 2**20:.0f} MiB >= 3x L2)"},
        "gpu_launches": len(PREFILL_CASES) * args.steps,
        "roofline": {"bound": "tensor",
                     "kernel": "w4_gemm_kernel M=%d K=%d N=%d" % PREFILL_CASES[dom],
                     "achieved": round(flops[dom] / (per[dom] / 1e3) / 1e12, 1), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(flops[dom] / (per[dom] / 1e3) / 1e12 / peak, 4),
                     "peak_kind": peak_kind + " bf16 cuBLAS burst", "traffic": None,
                     "mean_launch_us": round(per[dom] * 1e3, 2)},
        "per_case": [{"M": M, "K": K, "N": N, "us": round(t * 1e3, 2),
                      "TFLOPs": round(f / (t / 1e3) / 1e12, 1),
                      "dense_fp16_cublas_us": round(cb * 1e3, 2),
                      "reference_path_us": round(rf * 1e3, 2)}
                     for (M, K, N), t, f, cb, rf in zip(PREFILL_CASES, per, flops, cublas_ms, ref_ms)],
        "e2e": {"value": round(tot_flops * world * e_steps / (e_ms / 1e3) / 1e12, 2),
                "unit": "TFLOP/s",
                "h2d_bytes_per_step": sum(h.numel() * 2 for h in hx),
                "d2h_bytes_per_step": sum(h.numel() * 2 for h in hy),
                "path": "roofline_decoding_b200.w4_gemm per GEMM, pinned H2D x, D2H y, host sync"},
        "cpu_baseline": None,
        "clocks": clk,
    }
    return line


DECODE_PROMPT = 32   # random prompt ids, as the decode configuration states
DECODE_TOKENS = 256  # greedy tokens timed per run


def decode_cpu_baseline(model, prompt, seconds):
    """tok/s of the same model stepped on the host cores (oracle/decode_oracle.py).

    The reference's decode caller (scripts/decode_loop.py:107-124) restated in
    fp32 torch with every int4 linear on the reference's dequantise-then-matmul
    path in C; one warm-up token, then whole tokens for about `seconds`.
    """
    from oracle.decode_oracle import DecodeOracle

    ref = DecodeOracle(model)
    tok = int(prompt[0])
    ref.step(tok)  # warm the OpenMP pool and the pages
    n, t0 = 0, time.perf_counter()
    while n < 2 or (time.perf_counter() - t0 < seconds and n < 64):
        tok = int(torch_argmax(ref.step(tok)))
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(n / dt, 3), "unit": "tok/s", "cores": ref.cores, "kind": "port",
            "sample": f"{n} greedy tokens at positions 1..{n} in {dt:.1f} s: fp32 torch "
                      "Qwen2.5-1.5B-architecture step on the host, every int4 linear "
                      "dequantised to fp16 then fp32 GEMV (oracle/w4_oracle.c, OpenMP)"}


def torch_argmax(v):
    import torch

    return torch.argmax(v).item()


def run_decode(args, rank, world, local, cpu=True):
    """Batch-1 greedy decode of the Qwen2.5-1.5B architecture; record on rank 0."""
    import torch

    from roofline_decoding_b200.decode import W4DecodeModel

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    peak, peak_kind = measured_peaks()
    model = W4DecodeModel(device=device, seed=0, mode=args.decode_mode)
    model.capture()
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, model.cfg.vocab, (DECODE_PROMPT,), generator=g)
    steps = DECODE_TOKENS
    if DECODE_PROMPT + args.warmup + steps > model.cfg.max_seq:
        raise SystemExit("prompt + warmup + tokens exceed the 2048-token KV cache")

    def prefill():
        model.set_prompt(prompt)
        for _ in range(DECODE_PROMPT + args.warmup):  # untimed: prompt, then warm-up tokens
            model.graph.replay()

    prefill()
    torch.cuda.synchronize()
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        s_ev.record()
        for _ in range(steps):
            model.graph.replay()
        e_ev.record()
        torch.cuda.synchronize()
    ms = max_over_ranks([s_ev.elapsed_time(e_ev)], world)[0]
    tok_s = world * steps / (ms / 1e3)
    # the attention reads positions 0..pos: bytes at the mean position of the timed steps
    mean_seq = DECODE_PROMPT + args.warmup + (steps + 1) // 2
    step_bytes = model.bytes_per_step(seq_len=mean_seq)
    achieved = step_bytes * (steps / (ms / 1e3)) / 1e9

    # e2e: a host-driven loop that reads every token (like .item() per token)
    # and writes it back as the next step's input
    host_tok = torch.zeros((1,), dtype=torch.long).pin_memory()
    prefill()
    host_tok.copy_(model.token)
    torch.cuda.synchronize()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for _ in range(steps):
        model.token.copy_(host_tok, non_blocking=True)
        model.graph.replay()
        host_tok.copy_(model.token, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    e2.record()
    torch.cuda.synchronize()
    ms2 = max_over_ranks([s2.elapsed_time(e2)], world)[0]
    clk = clocks.summary()
    if rank != 0:
        del model
        torch.cuda.empty_cache()
        return None
    cpu_rec = None
    if cpu and world == 1 and not args.no_cpu_baseline:
        cpu_rec = decode_cpu_baseline(model, prompt, args.cpu_seconds)
    line = {
        "metric": "batch-1 greedy decode tok/s (W4A16 Qwen2.5-1.5B architecture, CUDA graph)",
        "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": round(ms / steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "w4a16 linears, bf16 activations/lm_head",
        "data": "synthetic (random-init seeded weights, 32 random prompt ids)",
        "config": {"workload": "Qwen2.5-1.5B architecture decode, 28 layers, hidden 1536, "
                               "int4 linears, tied bf16 lm_head 1536x151936, static KV 2048",
                   "prompt": DECODE_PROMPT, "tokens": steps},
        "parallelism": f"replicas{world}",
        "step": ("one persistent cooperative kernel (w4_decode_step)"
                 if args.decode_mode == "mega" else
                 "142 PDL-chained kernels (embed, 5 per layer, lm_head)"),
        "positions": f"{DECODE_PROMPT + args.warmup}..{DECODE_PROMPT + args.warmup + steps - 1}",
        "gpu_launches": model.launches_per_step() * steps,
        "roofline": {"bound": "hbm", "kernel": "decode step (all kernels)",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": None, "bytes_per_step": step_bytes,
                     "kv_positions_read": mean_seq,
                     "ceiling_tok_s": round(peak * 1e9 / step_bytes, 1)},
        "e2e": {"value": round(world * steps / (ms2 / 1e3), 2), "unit": "tok/s",
                "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8,
                "ms_per_step": round(ms2 / steps, 4),
                "path": "W4DecodeModel graph replay, token H2D + D2H and a host sync per step"},
        "cpu_baseline": cpu_rec,
        "clocks": clk,
    }
    del model
    torch.cuda.empty_cache()
    return line


def run_default(args, rank, world, local):
    """The sweep line with the large, decode and (N > 1) column-parallel records."""
    line = run_gemv_workload(args, rank, world, local, "sweep")
    if args.sweep_only:
        return line
    sub = {"large": run_gemv_workload(args, rank, world, local, "large", shard=False,
                                      cpu=False)}
    sub["decode"] = run_decode(args, rank, world, local)
    if world > 1:
        sub["column_parallel"] = run_gemv_workload(args, rank, world, local, "large",
                                                   shard=True, cpu=False)
    if rank != 0:
        return None
    for key in ("large", "column_parallel"):
        rec = sub.get(key)
        if rec is not None:  # the sub-records need no second copy of the shared fields
            for k in ("data", "dtype", "higher_is_better", "vs_baseline", "warmup"):
                rec.pop(k, None)
    if sub.get("column_parallel") is not None:
        one = sub["large"]["ms_per_step"]
        sub["column_parallel"]["one_gpu_ms_per_step"] = one
        sub["column_parallel"]["speedup_over_one_gpu"] = round(
            one / sub["column_parallel"]["ms_per_step"], 3)
    line.update(sub)
    return line


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["sweep", "gemm", "large", "decode", "prefill"],
                    default="sweep")
    ap.add_argument("--sweep-only", action="store_true",
                    help="default workload without the large/decode/column-parallel records")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--gather", choices=["peer", "nccl"], default="peer",
                    help="large workload on N>1 GPUs: all-gather fused into the GEMV (peer "
                         "stores over NVLink) or a separate NCCL all-gather")
    ap.add_argument("--decode-mode", choices=["mega", "fused"], default="fused",
                    help="decode workload: the step as one kernel or as 142 kernels")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":  # CPU only: no process group, rank 0 alone works
        world = int(os.environ.get("WORLD_SIZE", "1"))
        if world != args.gpus:
            raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
        run_reference(args, int(os.environ.get("RANK", "0")), world)
        return
    rank, world, local = dist_setup(args.gpus)
    try:
        if args.workload == "decode":
            line = run_decode(args, rank, world, local)
        elif args.workload == "prefill":
            line = run_prefill(args, rank, world, local)
        elif args.workload == "sweep":
            line = run_default(args, rank, world, local)
        else:
            line = run_gemv_workload(args, rank, world, local)
        if rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
