// w4_internal.h - declarations shared by the library's translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/w4b200.h"

namespace w4 {

// Records a failure message for w4_last_error() and returns the status.
int fail(int status, const char* fmt, ...);
// Converts a CUDA runtime error into W4_ERR_CUDA with a message.
int cuda_fail(cudaError_t e, const char* what);

// Per-device state filled by w4_init().
struct DeviceInfo {
  int sm_count = 0;
  int max_smem_optin = 0;  // bytes of dynamic shared memory a CTA may opt into
  int cc_major = 0, cc_minor = 0;
  int* err_word = nullptr;  // device address of the kernels' error word
};
const DeviceInfo& device_info(int device);
int current_device(int* dev);

// Launchers (no validation: the C ABI layer validates first).
cudaError_t launch_pack(const void* w, int w_dtype, int32_t* packed, void* scales, int K,
                        int N, int group_size, cudaStream_t stream);
cudaError_t launch_dequant(const int32_t* packed, const void* scales, void* out, int out_bf16,
                           int K, int N, cudaStream_t stream);

struct GemvLaunch {
  const void* x;
  const int32_t* packed;
  const void* scales;
  void* y;
  int x_bf16, y_bf16;
  int M, K, N;
  w4_gemv_config cfg;
  w4_fused_ops ops;  // zero for a plain GEMV
  const w4_peer_out* peer = nullptr;  // column-parallel: y gathered into every rank's buffer
};
size_t gemv_smem_bytes(int M, int K, int N, const w4_gemv_config& cfg);
// Column tiles covering N, and CTA columns of the launch (cfg.columns, or
// one per tile when 0 or not below the tile count).
int gemv_tiles(int N, const w4_gemv_config& cfg);
int gemv_columns(int N, const w4_gemv_config& cfg);
int gemv_validate_config(int M, int K, int N, const w4_gemv_config& cfg, const DeviceInfo& di);
int gemv_choose_config(int M, int K, int N, int split_k, int num_warps, const DeviceInfo& di,
                       w4_gemv_config* out);
int launch_gemv(const GemvLaunch& L, cudaStream_t stream);
// Launch plans (w4_gemv_plan_*): a prepared launch kept on the host.
int gemv_plan_create(const GemvLaunch& L, void** plan);
int gemv_plan_launch(const void* plan, const void* x_host, void* x, void* y, void* y_host,
                     cudaStream_t stream);
int gemv_plans_launch(const void* const* plans, int n, const void* x_host, void* x, void* y,
                      void* y_host, cudaStream_t stream);
void gemv_plan_destroy(void* plan);
// Times the tile candidates for (M, K, N) and returns the fastest (w4_tune.cu).
int gemv_tune(int M, int K, int N, int x_bf16, int y_bf16, int split_k, int num_warps,
              w4_gemv_config* out, float* best_us);
int gemv_init_device(const DeviceInfo& di);

// Decode-step kernels (w4_decode.cu).
int launch_decode_embed(const void* embed, int vocab, int hidden, const int64_t* prompt,
                        const int64_t* prompt_len, int64_t* token, const int64_t* pos, void* h,
                        int pdl, cudaStream_t stream);
int launch_decode_attention(const void* qkv, const void* cos_t, const void* sin_t,
                            const int64_t* pos, void* k_cache, void* v_cache, void* out, int heads,
                            int kv_heads, int max_seq, int pdl, cudaStream_t stream);
size_t lm_head_workspace_bytes();
int launch_lm_head_argmax(const void* h, const void* norm_w, float eps, const void* embed,
                          int vocab, int hidden, void* logits, int64_t* token, int64_t* pos,
                          void* workspace, int pdl, cudaStream_t stream);
int lm_head_argmax_static(const void* h, const void* norm_w, float eps, const void* embed,
                          int vocab, int hidden, void* logits, int64_t* token, int64_t* pos,
                          int pdl, cudaStream_t stream);
int decode_init_device(const DeviceInfo& di);
// The hidden sizes the lm_head kernel is built for (256, 512, 1024, 1536, 2048).
inline bool lm_head_hidden_supported(int hidden) {
  return hidden == 256 || hidden == 512 || hidden == 1024 || hidden == 1536 || hidden == 2048;
}

// tcgen05 W4A16 GEMM (w4_gemm.cu).
int gemm_init_device(const DeviceInfo& di);
int launch_gemm(const void* x, int x_bf16, const int32_t* packed, const void* scales, void* y,
                int y_bf16, int M, int K, int N, int split_k, cudaStream_t stream);

// Calibrated (GPTQ) packing, one 128-row block (w4_gptq.cu).
int gptq_init_device(const DeviceInfo& di);
int launch_gptq_block(const float* w, const float* u, int N, int32_t* packed, void* scales,
                      float* err, cudaStream_t stream);

// Whole-step persistent kernel (w4_mega.cu).
int mega_init_device(const DeviceInfo& di);
int decode_step_scratch_bytes(const w4_decode_model& m, size_t* bytes);
int launch_decode_step(const w4_decode_model& m, void* scratch, size_t scratch_bytes,
                       cudaStream_t stream);

// Tensor-map encoder resolved from the driver at init.
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled_fn();

}  // namespace w4
