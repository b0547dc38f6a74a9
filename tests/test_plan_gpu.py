"""Launch plans (GemvPlan, C ABI w4_gemv_plan_*) against the per-call entry point.

A plan prepares one layer's launch once; calling it must give exactly what
w4_matmul gives with the same tile (same kernel, same summation order), for
device buffers and for the host-buffer call that also copies x in and y out.
"""
import numpy as np
import pytest
import torch

from oracle import w4_oracle as o

pytestmark = pytest.mark.gpu

from roofline_decoding_b200 import kernels as K  # noqa: E402

DEV = "cuda"


@pytest.mark.parametrize("M,Kd,N,dt", [(1, 1536, 1536, torch.float16), (1, 8960, 1536, torch.bfloat16),
                                       (4, 4096, 1024, torch.float16), (16, 1024, 2816, torch.bfloat16)])
def test_plan_matches_w4_matmul(M, Kd, N, dt):
    p, s = K.pack_weights(torch.from_numpy(o.normal_weights(Kd, N, seed=Kd + N)).to(DEV))
    g = torch.Generator().manual_seed(M + Kd)
    plan = K.GemvPlan(p, s, M, dt, torch.float16)
    for step in range(3):
        x = torch.randn((M, Kd), generator=g).to(dt).to(DEV)
        want = K.w4_matmul(x, p, s, config=plan.config)
        got = plan(x)
        assert torch.equal(got, want), step
    # the host-buffer call: x copied in, y copied out, one C call
    hx = torch.randn((M, Kd), generator=g).to(dt).pin_memory()
    hy = torch.empty((M, N), dtype=torch.float16).pin_memory()
    xd = torch.empty((M, Kd), dtype=dt, device=DEV)
    yd = torch.empty((M, N), dtype=torch.float16, device=DEV)
    plan.launch_ptrs(hx.data_ptr(), xd.data_ptr(), yd.data_ptr(), hy.data_ptr(),
                     K._stream_ptr(xd.device))
    torch.cuda.synchronize()
    want = K.w4_matmul(hx.to(DEV), p, s, config=plan.config).cpu()
    assert torch.equal(hy, want)
    y_ref = o.gemv_reference(hx.float().numpy(), p.cpu().numpy(), s.cpu().numpy())
    np.testing.assert_allclose(hy.float().numpy(), y_ref, rtol=1e-2, atol=1e-2)
    assert K.device_error() == 0


def test_plan_rejects_wrong_inputs():
    p, s = K.pack_weights(torch.from_numpy(o.normal_weights(256, 64, seed=1)).to(DEV))
    plan = K.GemvPlan(p, s, 1, torch.float16)
    with pytest.raises(ValueError):
        plan(torch.zeros((1, 256), dtype=torch.bfloat16, device=DEV))
    with pytest.raises(ValueError):
        plan(torch.zeros((2, 256), dtype=torch.float16, device=DEV))
    with pytest.raises(ValueError):
        K.GemvPlan(p, s, 17, torch.float16)


def test_plan_batch_runs_every_plan_on_its_slices():
    """GemvPlan.batch: inputs back to back in one host buffer, one copy in, the
    GEMVs in order, one copy out; each slice equals that plan's own call."""
    shapes = [(1, 1536, 256, torch.float16), (1, 1024, 2816, torch.bfloat16),
              (2, 512, 1024, torch.float16)]
    plans, xs = [], []
    g = torch.Generator().manual_seed(5)
    for i, (M, Kd, N, dt) in enumerate(shapes):
        p, s = K.pack_weights(torch.from_numpy(o.normal_weights(Kd, N, seed=i)).to(DEV))
        plans.append(K.GemvPlan(p, s, M, dt, torch.float16, pdl=bool(i % 2)))
        xs.append(torch.randn((M, Kd), generator=g).to(dt))
    batch = K.GemvPlan.batch(plans)
    hx = torch.cat([x.view(torch.int16).reshape(-1) for x in xs]).pin_memory()
    hy = torch.empty((batch.y_elems,), dtype=torch.float16).pin_memory()
    xd = torch.empty_like(hx, device=DEV)
    yd = torch.empty_like(hy, device=DEV)
    for _ in range(2):
        batch.launch_ptrs(hx.data_ptr(), xd.data_ptr(), yd.data_ptr(), hy.data_ptr(),
                          K._stream_ptr(xd.device))
        torch.cuda.synchronize()
        off = 0
        for plan, x in zip(plans, xs):
            want = plan(x.to(DEV)).cpu().reshape(-1)
            assert torch.equal(hy[off:off + want.numel()], want)
            off += want.numel()
    assert K.device_error() == 0
