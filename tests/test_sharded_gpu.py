"""Column-parallel GEMV with the all-gather fused into the kernel, on 2 GPUs.

Two processes (one per GPU, NCCL for the handle exchange) run
w4_gemv_allgather: every rank's gathered y must equal, slice by slice and bit
for bit, the plain fused GEMV of each rank's columns with the same tile, and
stay right across calls (the output alternates between two buffers).
Skipped with fewer than two GPUs.
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, K, N, M, results):
    import datetime

    import torch.distributed as dist

    from roofline_decoding_b200 import kernels as Kn
    from roofline_decoding_b200.sharded import PeerGroup, ShardedW4Linear, shard_columns

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        g = torch.Generator(device="cpu").manual_seed(7)
        w = (torch.randn((K, N), generator=g) * 0.02).half().to(dev)
        packed, scales = Kn.pack_weights(w)
        peers = PeerGroup(device=dev)
        n_loc = N // world
        mine = shard_columns(packed, scales, rank, world, dev)
        # Every rank and both gathers must use one tile for the slices to compare
        # bit for bit, and a tuning run in each process could pick different
        # ones: fix the shard shape's tile (one column tile per CTA, which the
        # fused gather needs) before the first call.
        Kn._load_tuned_file()
        Kn._TUNE_CACHE[Kn._tune_key(dev, M, K, n_loc, torch.float16, torch.float16, None,
                                    None)] = (1, 8, 2, 1, 0)
        cfg = Kn.tuned_config(M, K, n_loc, torch.float16, torch.float16, None, None, dev,
                              streaming=False)
        ok = True
        for step in range(5):
            x = torch.randn((M, K), generator=torch.Generator().manual_seed(step)).half().to(dev)
            y = peers.gemv(x, *mine, "y", N, rank * n_loc, config=cfg).clone()
            torch.cuda.synchronize()
            for q in range(world):
                pq, sq = shard_columns(packed, scales, q, world, dev)
                want = Kn.w4_matmul(x, pq, sq, config=cfg)
                got = y[:, q * n_loc:(q + 1) * n_loc]
                ok &= bool(torch.equal(got, want))
        # the module path, against the NCCL gather of the same shards
        lin_p = ShardedW4Linear(packed, scales, device=dev, peers=peers, name="mod")
        lin_n = ShardedW4Linear(packed, scales, device=dev)
        x = torch.randn((1, K), generator=torch.Generator().manual_seed(99)).half().to(dev)
        ok &= bool(torch.equal(lin_p(x), lin_n(x)))
        err = Kn.device_error(rank)
        results[rank] = (ok, err)
        peers.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("K,N,M", [(1024, 4096, 1), (2048, 2048, 4)])
def test_gemv_allgather_two_gpus(K, N, M):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, K, N, M, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert results[0] == (True, 0) and results[1] == (True, 0), dict(results)
