"""Pins the CPU oracle to the reference: golden vectors made by the reference's own
pack_weights / reference_gemv (tests/golden/make_golden.py), the C restatement
against the numpy one, and the packer's numeric corner cases."""
import hashlib

import numpy as np
import pytest

from oracle import c_oracle
from oracle import w4_oracle as o


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def gen(K, N, kind, seed=0):
    return o.normal_weights(K, N, seed) if kind == "normal" else o.absmax_weights(K, N, seed)


@pytest.mark.parametrize("name", ["q_proj", "mlp_gate_up", "mlp_down", "kv_proj", "small_attn",
                                  "small_mlp", "ci_256x512", "absmax_q_proj", "absmax_mlp_gate",
                                  "absmax_mlp_down", "absmax_1024x2816"])
def test_numpy_pack_matches_reference_hashes(golden_hashes, name):
    c = golden_hashes["cases"][name]
    p, s = o.pack_weights(gen(c["K"], c["N"], c["kind"]), nan_as="cpu")
    assert sha(p) == c["packed_sha256"]
    assert sha(s) == c["scales_sha256"]


def test_c_pack_matches_reference_hash_4096x14336(golden_hashes):
    c = golden_hashes["cases"]["gemm_4096x14336"]
    p, s = c_oracle.pack(gen(c["K"], c["N"], c["kind"]), nan_as="cpu")
    assert sha(p) == c["packed_sha256"]
    assert sha(s) == c["scales_sha256"]


@pytest.mark.parametrize("name", ["large_8192x28672", "large_28672x8192", "vocab_8192x128256"])
def test_c_pack_matches_reference_chunk_hashes(golden_hashes, name):
    c = golden_hashes["chunked"][name]
    step = golden_hashes["chunk_n"]
    w = gen(c["K"], c["N"], c["kind"])
    p, s = c_oracle.pack(w, nan_as="cpu")
    for i, c0 in enumerate(range(0, c["N"], step)):
        assert sha(p[:, c0:c0 + step]) == c["packed_sha256"][i], f"chunk {i}"
        assert sha(s[:, c0:c0 + step]) == c["scales_sha256"][i], f"chunk {i}"


@pytest.mark.parametrize("case", ["normal_256x512", "absmax_128x64", "normal_1024x96", "edge"])
def test_pack_raw_cases_bit_exact(golden_small, case):
    w = golden_small[f"{case}/w"]
    p_ref, s_ref = golden_small[f"{case}/packed"], golden_small[f"{case}/scales"]
    for packer in (o.pack_weights, c_oracle.pack):
        p, s = packer(w, nan_as="cpu")
        np.testing.assert_array_equal(p, p_ref)
        np.testing.assert_array_equal(s.view(np.uint16), s_ref.view(np.uint16))


def test_edge_cases_cover_the_packer_corners(golden_small):
    """The edge fixture really exercises ties, zero/underflowing groups and NaN."""
    w = golden_small["edge/w"].astype(np.float32)
    s = golden_small["edge/scales"].astype(np.float32)
    p = golden_small["edge/packed"]
    q = o.unpack_nibbles(p)
    # column 0: s == 1, w in {.5, 1.5, 2.5, ...}: half to even
    assert s[0, 0] == 1.0
    expect = np.rint(w[:12, 0]) + 8
    np.testing.assert_array_equal(q[:12, 0], expect.astype(np.uint8))
    # column 1: all-zero groups -> scale 0 and NaN quotients -> the CPU reference's INT32_MIN
    assert (s[:, 1] == 0).all()
    assert (p[:, 1] == np.int32(-2 ** 31)).all()
    # column 2: one tiny value: scale underflows, the value saturates at 15 / 0
    assert s[0, 2] == 0 and q[5, 2] == 15 and q[130, 2] == 0


def test_cuda_nan_semantics_differ_only_in_nan_words(golden_small):
    """nan_as='cuda' (what the CUDA packer stores) differs from the CPU reference
    only in words that hold a NaN quotient; both dequantise to the same weights."""
    w = golden_small["edge/w"]
    p_cpu, s_cpu = o.pack_weights(w, nan_as="cpu")
    p_cuda, s_cuda = o.pack_weights(w, nan_as="cuda")
    np.testing.assert_array_equal(s_cpu.view(np.uint16), s_cuda.view(np.uint16))
    wf = w.astype(np.float32).reshape(2, 128, -1)
    with np.errstate(divide="ignore", invalid="ignore"):
        nanq = np.isnan(wf / s_cpu.astype(np.float32)[:, None, :]).reshape(256 // 8, 8, -1)
    nan_words = nanq.any(axis=1)
    assert nan_words.any()
    np.testing.assert_array_equal(p_cpu[~nan_words], p_cuda[~nan_words])
    # the NaN nibbles themselves hold 0 in the CUDA semantics
    q_cuda = o.unpack_nibbles(p_cuda)
    assert (q_cuda[nanq.reshape(256, -1)] == 0).all()
    d_cpu = o.dequantize_f32(p_cpu, s_cpu)
    d_cuda = o.dequantize_f32(p_cuda, s_cuda)
    finite = np.isfinite(d_cpu) & np.isfinite(d_cuda)
    np.testing.assert_array_equal(d_cpu[finite], d_cuda[finite])


def test_scale_is_division_path_independent():
    """torch divides a tensor by a CPU scalar exactly on the CPU but as a multiply
    by fp32(1/7) on CUDA; after the fp16 rounding of the scale the two agree
    for every finite fp16 amax, so the packer is device-independent."""
    h = np.arange(0, 0x7C00, dtype=np.uint16).view(np.float16).astype(np.float32)
    amax = np.maximum(h, np.float32(1e-8))
    a = (amax / np.float32(7.0)).astype(np.float16).view(np.uint16)
    b = (amax * np.float32(1.0 / 7.0)).astype(np.float16).view(np.uint16)
    np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("case", ["normal_256x512", "absmax_128x64", "normal_1024x96"])
@pytest.mark.parametrize("M", [1, 4])
@pytest.mark.parametrize("xdt", ["f16", "bf16"])
def test_gemv_reference_matches_golden(golden_small, case, M, xdt):
    p, s = golden_small[f"{case}/packed"], golden_small[f"{case}/scales"]
    x = golden_small[f"{case}/x_{xdt}_m{M}"]
    y_ref = golden_small[f"{case}/y_{xdt}_m{M}"]
    bf = xdt == "bf16"
    # reference_gemv rounds to fp16 (kernels.py:273); the bf16 golden stays fp32
    tol = dict(rtol=1e-5, atol=1e-5) if bf else dict(rtol=1e-3, atol=1e-4)
    y = o.gemv_reference(x, p, s, x_is_bf16_bits=bf)
    np.testing.assert_allclose(y, y_ref.astype(np.float32), **tol)
    yc = c_oracle.dequant_matmul(x, p, s, x_bf16=bf)
    np.testing.assert_allclose(yc, y_ref.astype(np.float32), **tol)
    # the exact (fp32-weight, float64) sum differs only by fp16 weight rounding
    ye = o.gemv_exact(x, p, s, x_is_bf16_bits=bf)
    np.testing.assert_allclose(ye, y_ref, rtol=1e-2, atol=1e-2)


def test_c_oracle_matches_numpy_oracle():
    w = o.absmax_weights(512, 384, 3)
    p, s = o.pack_weights(w)
    pc, sc = c_oracle.pack(w)
    np.testing.assert_array_equal(p, pc)
    np.testing.assert_array_equal(o.dequantize_fp16(p, s).view(np.uint16),
                                  c_oracle.dequant_fp16(p, s).view(np.uint16))
    x = o.activations(3, 512, 5)
    np.testing.assert_allclose(c_oracle.gemv_exact(x, p, s), o.gemv_exact(x, p, s),
                               rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("K,N", [(1536, 1536), (256, 512), (1024, 2816)])
def test_roundtrip_error_bounded(K, N):
    """tests/test_kernels.py:32-40: |w - dequant(pack(w))| < 0.15 on the absmax data."""
    w = o.absmax_weights(K, N, 0)
    p, s = o.pack_weights(w)
    assert p.shape == (K // 8, N) and s.shape == (K // 128, N)
    assert p.dtype == np.int32 and s.dtype == np.float16
    err = np.abs(w.astype(np.float32) - o.dequantize_fp16(p, s).astype(np.float32))
    assert err.max() < 0.15


def test_bf16_rounding_helper():
    vals = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38, 1e-40, 0.0, -0.0],
                    dtype=np.float32)
    bits = o.f32_to_bf16_bits(vals)
    back = o.bf16_bits_to_f32(bits)
    # 1 + 2^-8 is a tie between 1 and 1 + 2^-7 -> even (1.0)
    assert back[1] == 1.0
    assert back[2] == np.float32(1.015625)  # 1 + 3*2^-8 rounds up to 1 + 2^-6
    assert back[3] == -2.5 and back[6] == 0.0
