"""The tcgen05 W4A16 GEMM (w4_gemm, the prefill rows of W4Linear) on the GPU.

fp16 activations: the reference's prefill path is dequantize_v1 (fp16
weights fp16((q - 8) * s)) then an fp32 matmul (scripts/decode_loop.py:51-55);
the kernel multiplies the same fp16 weights on the tensor cores with fp32
accumulation, so it matches the oracle's dequantise-then-fp32-matmul up to
the summation order (tight bar), and within the required rtol = atol = 1e-2.
bf16 activations use bf16 weights (one rounding of the fp32 product).
"""
import numpy as np
import pytest
import torch

from oracle import w4_oracle as o

pytestmark = pytest.mark.gpu

from roofline_decoding_b200 import W4Linear, kernels as Kn  # noqa: E402


def _case(M, K, N, seed=0, x_dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn((K, N), generator=g) * 0.02).half()
    x = torch.randn((M, K), generator=g).to(x_dtype)
    packed, scales = Kn.pack_weights(w.cuda())
    return x, packed, scales


def _want(x, packed, scales, bf16_weights=False):
    """Oracle: fp16 (or bf16) dequantised weights, fp32 matmul, in numpy."""
    wd = o.dequantize_f32(packed.cpu().numpy(), scales.cpu().numpy())  # (q - 8) * s in fp32
    wt = torch.from_numpy(wd)
    wt = wt.bfloat16().float() if bf16_weights else wt.half().float()
    return x.float() @ wt


@pytest.mark.parametrize("M,K,N", [(128, 128, 128), (17, 256, 256), (300, 1024, 384),
                                   (1024, 1536, 1536), (1, 512, 128), (200, 4096, 1024),
                                   # grids of >= 148 256-wide tiles: the 256-column tile,
                                   # the second with a half-filled last tile (N % 256 = 128)
                                   (2048, 512, 4864), (4000, 256, 2432),
                                   # 128-column tiles of 256 rows (two accumulators)
                                   (5700, 128, 896), (600, 384, 640)])
def test_gemm_fp16_matches_oracle(M, K, N):
    x, packed, scales = _case(M, K, N, seed=M + K)
    y = Kn.w4_gemm(x.cuda(), packed, scales).float().cpu()
    want = _want(x, packed, scales)
    # tight: the same fp16 products, fp32 sums in another order, one fp16 rounding
    assert torch.allclose(y, want.half().float(), rtol=4e-3, atol=4e-3), \
        (y - want).abs().max().item()
    assert torch.allclose(y, want, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("M,K,N", [(256, 512, 256), (129, 2048, 640)])
def test_gemm_bf16_matches_oracle(M, K, N):
    x, packed, scales = _case(M, K, N, seed=3, x_dtype=torch.bfloat16)
    y = Kn.w4_gemm(x.cuda(), packed, scales).float().cpu()
    want = _want(x, packed, scales, bf16_weights=True)
    assert torch.allclose(y, want, rtol=2e-2, atol=2e-2), (y - want).abs().max().item()


def test_gemm_is_deterministic_and_ragged_rows_are_untouched():
    x, packed, scales = _case(130, 512, 256, seed=9)
    xd = x.cuda()
    out = torch.full((131, 256), 7.0, dtype=torch.float16, device="cuda")
    a = Kn.w4_gemm(xd, packed, scales)
    b = Kn.w4_gemm(xd, packed, scales)
    assert torch.equal(a, b)
    Kn.w4_gemm(xd, packed, scales, out=out[:130])
    assert torch.equal(out[:130], a)
    assert torch.all(out[130] == 7.0)  # rows past M are never written
    assert Kn.device_error() == 0


def test_w4linear_prefill_uses_the_gemm_and_matches_dense():
    torch.manual_seed(0)
    lin = torch.nn.Linear(1024, 768, bias=True).half().cuda()
    q = W4Linear(lin)
    x = torch.randn((3, 100, 1024), device="cuda").half()
    y = q(x)
    assert y.shape == (3, 100, 768) and y.dtype == torch.float16
    w = Kn.dequantize_v1(q.packed, q.scales).float()
    want = (x.reshape(-1, 1024).float() @ w + q.bias.float()).half().reshape(3, 100, 768)
    assert torch.allclose(y.float(), want.float(), rtol=1e-2, atol=1e-2)


def test_gemm_rejects_bad_shapes():
    x, packed, scales = _case(64, 256, 256)
    with pytest.raises(ValueError):
        Kn.w4_gemm(x.cuda()[:, :128], packed, scales)
    p2, s2 = Kn.pack_weights((torch.randn(256, 200) * 0.02).half().cuda())
    with pytest.raises(ValueError):
        Kn.w4_gemm(x.cuda(), p2, s2)


@pytest.mark.parametrize("M,K,N", [(300, 1024, 384), (129, 2048, 640), (100, 512, 256),
                                   (1024, 1536, 1536)])
@pytest.mark.parametrize("split_k", [2, 3, 5, 8])
def test_gemm_k_slices_match_oracle(M, K, N, split_k):
    """K cut into slices (128 x 256 tiles, a cluster per tile, partials summed
    over DSMEM in rank order), including slice counts that do not divide the
    64-k stages and a last tile half outside N."""
    x, packed, scales = _case(M, K, N, seed=M + split_k)
    y = Kn.w4_gemm(x.cuda(), packed, scales, split_k=split_k).float().cpu()
    want = _want(x, packed, scales)
    assert torch.allclose(y, want.half().float(), rtol=4e-3, atol=4e-3), \
        (y - want).abs().max().item()
    y2 = Kn.w4_gemm(x.cuda(), packed, scales, split_k=split_k).float().cpu()
    assert torch.equal(y, y2)  # a fixed summation order
    assert Kn.device_error() == 0


def test_gemm_k_slices_bf16():
    x, packed, scales = _case(257, 2048, 512, seed=4, x_dtype=torch.bfloat16)
    y = Kn.w4_gemm(x.cuda(), packed, scales, split_k=4).float().cpu()
    want = _want(x, packed, scales, bf16_weights=True)
    assert torch.allclose(y, want, rtol=2e-2, atol=2e-2), (y - want).abs().max().item()


@pytest.mark.parametrize("M,K,N", [
    (512, 4096, 1536),   # 24 tiles of 256 x 128, fewer than the SMs: one launch
    (1000, 512, 9728),   # 152 tiles of 256 x 256: 148 in one launch, 4 in a K-sliced second
])
def test_gemm_library_split_choices_match_oracle(M, K, N):
    x, packed, scales = _case(M, K, N, seed=K)
    y = Kn.w4_gemm(x.cuda(), packed, scales).float().cpu()
    want = _want(x, packed, scales)
    assert torch.allclose(y, want.half().float(), rtol=4e-3, atol=4e-3), \
        (y - want).abs().max().item()
    assert Kn.device_error() == 0


def test_gemm_prefill_shape_remainder_launch_rows():
    """2048 x 4096 x 14336 (the prefill workload): 444 tiles in the first
    launch, the last 4 in a K-sliced second one; the rows of the last tile row
    (both launches) and a band of the first against the oracle."""
    M, K, N = 2048, 4096, 14336
    x, packed, scales = _case(M, K, N, seed=11)
    y = Kn.w4_gemm(x.cuda(), packed, scales).float().cpu()
    for rows in (slice(1792, 2048), slice(0, 64)):
        want = _want(x[rows], packed, scales)
        assert torch.allclose(y[rows], want.half().float(), rtol=4e-3, atol=4e-3), \
            (y[rows] - want).abs().max().item()
    assert Kn.device_error() == 0
