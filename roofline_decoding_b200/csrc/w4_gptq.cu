// w4_gptq.cu - calibrated int4 packing (GPTQ), one 128-row block per launch.
//
// The reference names "Calibrated (GPTQ-style) scales" as its next step
// (devto_article.md:71) and keeps the packed format of
// src/roofline/kernels.py:24-47. This kernel is the sequential part of GPTQ
// (Frantar et al., 2022, Algorithm 1) for one block of 128 rows of W [K, N]
// (K = in-features), which is also one quantisation group:
//   s      = fp16(max|w| / 7) over the block's error-compensated rows;
//   row i  : q = clamp(rint(w_i / s) + 8, 0, 15), err_i = (w_i - (q-8) s) / U_ii,
//            rows j > i of the block: w_j -= U_ij * err_i;
// where U is the upper Cholesky factor of the conditioned inverse Hessian.
// The host applies the lazy batch update to the later blocks with one GEMM
// (W[b1:] -= U[b0:b1, b1:]^T @ err) and factors the Hessian.
//
// Layout: one thread per output column n; the block's 128 values of that
// column live in shared memory as w_s[row][thread] (consecutive threads on
// consecutive banks) and the block of U in shared memory, read as a broadcast.
// Arithmetic: IEEE fp32, the update as a rounded product then a rounded
// subtraction (no fused multiply-add), the same operations in the same order
// as the float32 oracle, so one block is reproducible bit for bit.
#include "w4_internal.h"

#include <cuda_fp16.h>

namespace w4 {

namespace {

constexpr int kGptqBlock = 128;    // rows per block = the quantisation group
constexpr int kGptqThreads = 128;  // columns per CTA

__global__ void __launch_bounds__(kGptqThreads)
    gptq_block_kernel(const float* __restrict__ w, const float* __restrict__ u, int N,
                      int32_t* __restrict__ packed, __half* __restrict__ scales,
                      float* __restrict__ err) {
  extern __shared__ float smem[];
  float* u_s = smem;                              // [128][128] U block (row-major)
  float* w_s = smem + kGptqBlock * kGptqBlock;    // [128 rows][kGptqThreads columns]
  const int t = threadIdx.x;
  const int n = blockIdx.x * kGptqThreads + t;
  const bool live = n < N;

  for (int i = t; i < kGptqBlock * kGptqBlock; i += kGptqThreads) u_s[i] = u[i];
  float amax = 0.f;
  bool has_nan = false;
  for (int r = 0; r < kGptqBlock; ++r) {
    const float v = live ? w[(size_t)r * N + n] : 0.f;
    w_s[r * kGptqThreads + t] = v;
    has_nan |= isnan(v);
    amax = fmaxf(amax, fabsf(v));
  }
  __syncthreads();
  if (!live) return;  // no barrier follows

  // The group scale of the pack_weights recipe, on the compensated weights.
  amax = has_nan ? __int_as_float(0x7fc00000) : fmaxf(amax, 1e-8f);
  const __half s_h = __float2half_rn(__fdiv_rn(amax, 7.0f));
  scales[n] = s_h;
  const float s = __half2float(s_h);

  uint32_t word = 0;
  for (int i = 0; i < kGptqBlock; ++i) {
    const float wi = w_s[i * kGptqThreads + t];
    float q = rintf(__fdiv_rn(wi, s)) + 8.0f;
    q = isnan(q) ? 0.f : fminf(fmaxf(q, 0.f), 15.f);
    const float wq = __fmul_rn(q - 8.0f, s);
    const float e = __fdiv_rn(__fsub_rn(wi, wq), u_s[i * kGptqBlock + i]);
    err[(size_t)i * N + n] = e;
    word |= static_cast<uint32_t>(q) << (4 * (i & 7));
    if ((i & 7) == 7) {
      packed[(size_t)(i >> 3) * N + n] = static_cast<int32_t>(word);
      word = 0;
    }
    const float* ui = u_s + i * kGptqBlock;
    for (int j = i + 1; j < kGptqBlock; ++j) {
      float& wj = w_s[j * kGptqThreads + t];
      wj = __fsub_rn(wj, __fmul_rn(ui[j], e));
    }
  }
}

}  // namespace

size_t gptq_smem_bytes() {
  return (size_t)(kGptqBlock * kGptqBlock + kGptqBlock * kGptqThreads) * sizeof(float);
}

int gptq_init_device(const DeviceInfo& di) {
  if (gptq_smem_bytes() > (size_t)di.max_smem_optin)
    return fail(W4_ERR_UNSUPPORTED, "GPTQ block needs %zu B of shared memory", gptq_smem_bytes());
  cudaError_t e = cudaFuncSetAttribute(gptq_block_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)gptq_smem_bytes());
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gptq smem)");
  e = cudaFuncSetAttribute(gptq_block_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gptq carveout)");
  return W4_OK;
}

int launch_gptq_block(const float* w, const float* u, int N, int32_t* packed, void* scales,
                      float* err, cudaStream_t stream) {
  const unsigned blocks = (unsigned)((N + kGptqThreads - 1) / kGptqThreads);
  gptq_block_kernel<<<blocks, kGptqThreads, gptq_smem_bytes(), stream>>>(
      w, u, N, packed, static_cast<__half*>(scales), err);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gptq block launch");
  return W4_OK;
}

}  // namespace w4
