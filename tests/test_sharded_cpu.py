"""Column-parallel sharding and gather logic on CPU gloo ranks (world size 2 and 4).

The per-rank compute is the oracle's dense restatement here (the CUDA kernel
needs a GPU); what is under test is the host logic: column ranges, shard
repacking, bias slicing and the all-gather assembly, against the unsharded
oracle result.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import w4_oracle as o


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def oracle_matmul(x2, packed, scales, out_dtype=torch.float16):
    y = o.gemv_exact(x2.float().numpy().astype(np.float16), packed.numpy(), scales.numpy())
    return torch.from_numpy(y.astype(np.float32)).to(out_dtype)


def _worker(rank, world, port, K, N, M, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from roofline_decoding_b200.sharded import ShardedW4Linear, column_range

        w = o.normal_weights(K, N, seed=1)
        p, s = o.pack_weights(w)
        bias = torch.from_numpy((np.arange(N) % 7).astype(np.float16) * 0.01)
        lin = ShardedW4Linear(torch.from_numpy(p), torch.from_numpy(s), bias=bias,
                              matmul=oracle_matmul)
        c0, c1 = column_range(N, rank, world)
        assert lin.packed.shape == (K // 8, c1 - c0) and lin.packed.is_contiguous()
        assert torch.equal(lin.packed, torch.from_numpy(p[:, c0:c1]))
        x = torch.from_numpy(o.activations(M, K, seed=2))
        y = lin(x)
        y_ref = o.gemv_exact(o.activations(M, K, seed=2), p, s) + bias.float().numpy()
        np.testing.assert_allclose(y.float().numpy(), y_ref, rtol=2e-3, atol=2e-3)
        q.put((rank, None))
    except Exception as e:  # report to the parent instead of hanging the group
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,M", [(2, 1), (2, 3), (4, 1)])
def test_sharded_matches_unsharded(world, M):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 256, 512, M, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    errors = [e for _, e in results if e]
    assert not errors, errors


def test_column_range_rules():
    from roofline_decoding_b200.sharded import column_range

    assert column_range(28672, 3, 8) == (3 * 3584, 4 * 3584)
    assert column_range(128256, 7, 8) == (7 * 16032, 128256)
    with pytest.raises(ValueError):
        column_range(100, 0, 3)
    with pytest.raises(ValueError):
        column_range(24, 0, 8)  # 3 columns per rank: not a multiple of 8
