"""A bounded wait that runs out: the gathered GEMV when a peer never arrives.

w4_gemv_allgather's last CTA on a rank publishes its epoch to every rank and
then waits, for at most one second, for every rank's epoch to arrive. Here one
process on one GPU plays rank 0 of a world of 2 whose rank 1 never runs: its
flag words and output buffers are local memory that nobody else writes. The
wait must give up after its bound, the kernel must return (no hang, no
fault), the device error word must read 6 (a peer's flag did not arrive), and
rank 0's own slice must still have been stored into both ranks' buffers.
The context stays usable: a plain GEMV runs right after.
"""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

from roofline_decoding_b200 import _lib  # noqa: E402
from roofline_decoding_b200 import kernels as Kn  # noqa: E402

DEV = "cuda"
K_ERR_PEER_WAIT = 6


def test_peer_flag_wait_times_out_and_reports():
    lib = _lib.load()
    K, n_loc, world = 1024, 256, 2
    g = torch.Generator(device="cpu").manual_seed(0)
    w = (0.02 * torch.randn((K, n_loc), generator=g)).half().to(DEV)
    packed, scales = Kn.pack_weights(w)
    x = torch.randn((1, K), generator=g).half().to(DEV)
    cfg = Kn.default_config(1, K, n_loc)
    assert Kn.device_error() == 0
    # rank q's buffers: y[parity][q] [1, world * n_loc]; flag words + state words
    ys = [[torch.zeros((1, world * n_loc), dtype=torch.float16, device=DEV) for _ in range(world)]
          for _ in range(2)]
    flag_region = [torch.zeros((64,), dtype=torch.int32, device=DEV) for _ in range(world)]
    po = _lib.PeerOut()
    po.world, po.rank, po.n_full, po.col_off = world, 0, world * n_loc, 0
    for b in range(2):
        for q in range(world):
            po.y[b][q] = ys[b][q].data_ptr()
    for q in range(world):
        po.flags[q] = flag_region[q].data_ptr()
    po.state = flag_region[0].data_ptr() + 128  # rank 0's state words, as PeerGroup lays them out
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    import ctypes

    _lib.check(lib.w4_gemv_allgather(x.data_ptr(), _lib.W4_F16, packed.data_ptr(),
                                     scales.data_ptr(), _lib.W4_F16, 1, K, n_loc,
                                     ctypes.byref(cfg), ctypes.byref(po),
                                     torch.cuda.current_stream().cuda_stream),
               "w4_gemv_allgather")
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert 0.9 <= waited < 30.0, waited  # the one-second bound, then the kernel returned
    assert Kn.device_error() == K_ERR_PEER_WAIT
    assert Kn.device_error() == 0  # read and cleared
    # the first call is epoch 1: parity 1; rank 0 published to both ranks' flag words
    assert int(flag_region[0][0].item()) == 1 and int(flag_region[1][0].item()) == 1
    assert int(flag_region[1][1].item()) == 0  # rank 1 never arrived
    state = flag_region[0][32:34].tolist()
    assert state == [1, 0], state  # epoch of the last call, CTA counter reset
    want = Kn.w4_matmul(x, packed, scales, config=cfg)
    for q in range(world):
        assert torch.equal(ys[1][q][:, :n_loc], want), q
        assert not ys[0][q].any()
    # the context is still usable
    y2 = Kn.w4_matmul(x, packed, scales, config=cfg)
    torch.cuda.synchronize()
    assert torch.equal(y2, want) and Kn.device_error() == 0
