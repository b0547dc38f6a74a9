"""Roofline accounting: the reference's tests/test_roofline.py re-targeted at this
package, plus this build's byte accounting (per-GEMV and per-decode-step)."""
import pytest

from roofline_decoding_b200.roofline import (ORCH_FUSION, QWEN_15B, achieved_bandwidth_percent,
                                             bytes_per_param, ceilings_table,
                                             count_decoder_params, decode_ceiling,
                                             decode_step_bytes, gemv_bytes, kv_bytes_per_token,
                                             weight_bytes_per_token)


class TestBytesPerParam:
    def test_known_sizes(self):
        assert bytes_per_param("bf16") == 2.0
        assert bytes_per_param("int8") == 1.0
        assert bytes_per_param("int4") == 0.5

    def test_unknown_raises(self):
        with pytest.raises(KeyError):
            bytes_per_param("fp32")


class TestParamCounts:
    def test_qwen_totals(self):
        c = count_decoder_params(QWEN_15B)
        assert c["head"] == 0
        assert c["embed"] == 151936 * 1536
        assert 0.10 < c["embed"] / c["total"] < 0.20
        assert 1.3e9 < c["total"] < 1.7e9

    def test_orch_totals(self):
        c = count_decoder_params(ORCH_FUSION)
        assert c["head"] == 2103 * 1024
        assert c["embed"] == 2103 * 1024
        assert 2.5e8 < c["total"] < 3.0e8

    def test_gqa_saves_kv_params(self):
        full = dict(QWEN_15B, kv_heads=12)
        gqa = dict(QWEN_15B, kv_heads=2)
        assert count_decoder_params(gqa)["decoder"] < count_decoder_params(full)["decoder"]

    def test_non_embedding_excludes_embed_and_head(self):
        c = count_decoder_params(QWEN_15B)
        assert c["non_embedding"] == c["total"] - c["embed"] - c["head"]


class TestWeightBytes:
    def test_bf16_int4_ratio(self):
        assert weight_bytes_per_token(QWEN_15B, "bf16") / weight_bytes_per_token(
            QWEN_15B, "int4") == pytest.approx(4.0)

    def test_qwen_bf16_gb(self):
        assert 2.6e9 < weight_bytes_per_token(QWEN_15B, "bf16") < 3.4e9

    def test_orch_int4_mb(self):
        assert 120e6 < weight_bytes_per_token(ORCH_FUSION, "int4") < 150e6


class TestKVBytes:
    def test_scales_with_seq_len(self):
        a = kv_bytes_per_token(QWEN_15B, "bf16", seq_len=1024)
        b = kv_bytes_per_token(QWEN_15B, "bf16", seq_len=2048)
        assert b == 2 * a

    def test_kv_small_vs_weights(self):
        kv = kv_bytes_per_token(QWEN_15B, "bf16", seq_len=2048)
        assert kv / weight_bytes_per_token(QWEN_15B, "bf16") < 0.15


class TestCeilings:
    def test_int4_ceiling_4x_bf16(self):
        a = decode_ceiling(QWEN_15B, "bf16", 300.0)
        b = decode_ceiling(QWEN_15B, "int4", 300.0)
        assert b.ceiling_tok_s / a.ceiling_tok_s == pytest.approx(4.0)

    def test_orch_faster_than_qwen(self):
        a = decode_ceiling(QWEN_15B, "int4", 300.0)
        b = decode_ceiling(ORCH_FUSION, "int4", 300.0)
        assert 4.5 < b.ceiling_tok_s / a.ceiling_tok_s < 6.5

    def test_table_shape(self):
        rows = ceilings_table(300.0)
        assert len(rows) == 6
        assert all(r["ceiling_tok_s"] > 0 for r in rows)


class TestAchievedPercent:
    def test_half_roofline(self):
        out = achieved_bandwidth_percent(50.0, 3.0, 0.0, 300.0)
        assert out["achieved_gbs"] == pytest.approx(150.0)
        assert out["percent_of_roofline"] == pytest.approx(50.0)

    def test_never_exceeds_100_legitimately(self):
        out = achieved_bandwidth_percent(200.0, 3.0, 0.0, 300.0)
        assert out["percent_of_roofline"] == pytest.approx(200.0)


class TestAlgorithmicBytes:
    @pytest.mark.parametrize("K,N,expect", [
        (1536, 1536, 1_222_656), (1536, 8960, 7_117_312), (1536, 256, 206_336),
        (1024, 1024, 544_768), (1024, 2816, 1_494_528), (8192, 28672, 121_184_256),
        (8192, 128256, 542_026_240), (4096, 14336, 30_314_496)])
    def test_gemv_bytes(self, K, N, expect):
        assert gemv_bytes(1, K, N) == expect

    def test_gemv_bytes_grow_with_rows(self):
        assert gemv_bytes(16, 4096, 14336) - gemv_bytes(1, 4096, 14336) == 15 * 2 * (4096 + 14336)

    def test_decode_step_bytes(self):
        d = decode_step_bytes(QWEN_15B, seq_len=2048)
        assert d["w4_packed"] == 655_097_856
        assert d["w4_scales"] == 20_471_808
        assert d["lm_head"] == 466_747_392
        assert d["biases"] == 114_688
        assert d["norms"] == 175_104
        assert d["embed_row"] == 3_072
        assert d["kv_read"] == 58_720_256
        assert d["total"] == 1_201_330_176

    def test_decode_kv_linear_in_positions(self):
        a = decode_step_bytes(QWEN_15B, seq_len=100)["kv_read"]
        b = decode_step_bytes(QWEN_15B, seq_len=200)["kv_read"]
        assert b == 2 * a == 2 * 28_672 * 100


@pytest.mark.gpu
def test_copy_bandwidth_in_b200_range():
    from roofline_decoding_b200.roofline import measure_copy_bandwidth_gbs

    bw = measure_copy_bandwidth_gbs(n_bytes=1 << 30, iters=5)
    assert 4000.0 < bw < 9000.0  # B200 HBM3e, measured ~6.45 TB/s on this pool
