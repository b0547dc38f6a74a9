"""B200-native (sm_100a) W4A16 dequantise + GEMV library.

Keeps the Python surface of the reference's hot path (roofline/kernels.py and
scripts/decode_loop.py): pack_weights, dequantize_v1, gemv_v2, gemv_v3,
reference_gemv, W4Linear, swap_linears, weight_bytes_int4, plus the roofline
helpers of roofline/roofline.py, and the calibrated (GPTQ) packing the
reference lists as its next step. Compute goes through libw4b200.so's C ABI.
"""
from .kernels import (GROUP_SIZE, _TUNE_CACHE, GemvPlan, default_config, dequantize_v1, device_error,
                      gemv_v2, gemv_v3, pack_weights, reference_gemv, save_tuned_configs,
                      tuned_config, w4_gemm, w4_matmul)
from .calibrate import accumulate_hessian, calibrate_linears, gptq_pack
from .linear import W4Linear, swap_linears, weight_bytes_int4
from .roofline import (ORCH_FUSION, QWEN_15B, achieved_bandwidth_percent, ceilings_table,
                       decode_ceiling, gemv_bytes, measure_copy_bandwidth_gbs)

__version__ = "1.0.0"
__all__ = [
    "GROUP_SIZE", "_TUNE_CACHE", "GemvPlan", "default_config", "dequantize_v1", "device_error", "gemv_v2",
    "gemv_v3", "pack_weights", "reference_gemv", "save_tuned_configs", "tuned_config",
    "w4_gemm", "w4_matmul", "W4Linear", "swap_linears", "weight_bytes_int4", "ORCH_FUSION", "QWEN_15B",
    "achieved_bandwidth_percent", "ceilings_table", "decode_ceiling", "gemv_bytes",
    "measure_copy_bandwidth_gbs", "accumulate_hessian", "calibrate_linears", "gptq_pack",
]
