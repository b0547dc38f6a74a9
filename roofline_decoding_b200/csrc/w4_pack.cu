// w4_pack.cu - int4 packer and v1 dequantiser.
//
// pack:    restates roofline/kernels.py:24-47 (pack_weights) on the GPU, bit
//          for bit: amax per (group, column) clamped at 1e-8, s = fp16(amax/7),
//          q = clamp(round_half_even(w / s) + 8, 0, 15), nibble i of word j
//          holds row 8j + i.
// dequant: restates roofline/kernels.py:50-74 (_dequant_kernel): the product
//          (q - 8) * s in fp32, rounded once to the output type.
#include "w4_internal.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace w4 {

__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(float v) { return v; }

// One thread per (group, column). Consecutive threads take consecutive
// columns, so every row read and word written is coalesced across the warp.
template <typename TW>
__global__ void __launch_bounds__(256) pack_kernel(const TW* __restrict__ w,
                                                   int32_t* __restrict__ packed,
                                                   __half* __restrict__ scales, int K, int N,
                                                   int group_size) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int groups = K / group_size;
  if (idx >= (long long)groups * N) return;
  const int n = (int)(idx % N);
  const int grp = (int)(idx / N);
  const TW* col = w + (size_t)grp * group_size * N + n;

  // amax = max |w| over the group; torch.amax propagates NaN.
  float amax = 0.f;
  bool has_nan = false;
  for (int r = 0; r < group_size; ++r) {
    const float v = to_f32(col[(size_t)r * N]);
    has_nan |= isnan(v);
    amax = fmaxf(amax, fabsf(v));
  }
  amax = has_nan ? __int_as_float(0x7fc00000) : fmaxf(amax, 1e-8f);  // .clamp(min=1e-8)
  // (amax / 7.0).to(float16): fp32 IEEE division, then round-to-nearest-even.
  // For every finite fp16 amax this equals amax * fp32(1/7) after the fp16
  // rounding, so the CPU and CUDA code paths of torch give the same scale.
  const __half s_h = __float2half_rn(__fdiv_rn(amax, 7.0f));
  scales[(size_t)grp * N + n] = s_h;
  const float s = __half2float(s_h);

  for (int j = 0; j < group_size / 8; ++j) {
    uint32_t word = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float v = to_f32(col[(size_t)(8 * j + i) * N]);
      // torch.round is round-half-even (rintf); fp32 / fp16 promotes to fp32.
      float q = rintf(__fdiv_rn(v, s)) + 8.0f;
      // clamp(0, 15) keeps NaN, and the int32 cast of NaN on a CUDA device is
      // 0; +-inf (s == 0, w != 0) clamp to 15 / 0 like the reference.
      q = isnan(q) ? 0.f : fminf(fmaxf(q, 0.f), 15.f);
      word |= static_cast<uint32_t>(q) << (4 * i);
    }
    packed[(size_t)(grp * (group_size / 8) + j) * N + n] = static_cast<int32_t>(word);
  }
}

cudaError_t launch_pack(const void* w, int w_dtype, int32_t* packed, void* scales, int K,
                        int N, int group_size, cudaStream_t stream) {
  const long long work = (long long)(K / group_size) * N;
  const int threads = 256;
  const long long blocks = (work + threads - 1) / threads;
  if (blocks == 0) return cudaSuccess;
  __half* sc = static_cast<__half*>(scales);
  if (w_dtype == W4_PACK_BF16)
    pack_kernel<<<(unsigned)blocks, threads, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(w), packed, sc, K, N, group_size);
  else if (w_dtype == W4_PACK_F32)
    pack_kernel<<<(unsigned)blocks, threads, 0, stream>>>(static_cast<const float*>(w), packed,
                                                         sc, K, N, group_size);
  else
    pack_kernel<<<(unsigned)blocks, threads, 0, stream>>>(static_cast<const __half*>(w), packed,
                                                         sc, K, N, group_size);
  return cudaGetLastError();
}

// Each thread expands one packed word row segment of 8 columns: reads two
// 16-byte packed vectors plus 16 bytes of scales and writes 8 rows x 16 bytes.
template <bool kBF16>
__global__ void __launch_bounds__(256) dequant_kernel(const int32_t* __restrict__ packed,
                                                      const __half* __restrict__ scales,
                                                      void* __restrict__ out, int K, int N) {
  const int n8 = N / 8;  // N % 8 == 0 is a precondition
  const long long total = (long long)(K / 8) * n8;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int k8 = (int)(idx / n8);
    const int c = (int)(idx % n8) * 8;
    const int4* src = reinterpret_cast<const int4*>(packed + (size_t)k8 * N + c);
    const int4 p0 = __ldg(src), p1 = __ldg(src + 1);
    const uint32_t words[8] = {(uint32_t)p0.x, (uint32_t)p0.y, (uint32_t)p0.z, (uint32_t)p0.w,
                               (uint32_t)p1.x, (uint32_t)p1.y, (uint32_t)p1.z, (uint32_t)p1.w};
    const int grp = (k8 * 8) / 128;
    const uint4 sv = __ldg(reinterpret_cast<const uint4*>(scales + (size_t)grp * N + c));
    const __half* sh = reinterpret_cast<const __half*>(&sv);
    float s[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i] = __half2float(sh[i]);
#pragma unroll
    for (int nib = 0; nib < 8; ++nib) {
      uint4 o;
      uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const float a = (float)((int)((words[2 * p] >> (4 * nib)) & 0xF) - 8) * s[2 * p];
        const float b = (float)((int)((words[2 * p + 1] >> (4 * nib)) & 0xF) - 8) * s[2 * p + 1];
        if constexpr (kBF16) {
          const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
          ow[p] = *reinterpret_cast<const uint32_t*>(&v);
        } else {
          const __half2 v = __floats2half2_rn(a, b);
          ow[p] = *reinterpret_cast<const uint32_t*>(&v);
        }
      }
      const size_t k = (size_t)k8 * 8 + nib;
      *reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + k * N + c) = o;
    }
  }
}

cudaError_t launch_dequant(const int32_t* packed, const void* scales, void* out, int out_bf16,
                           int K, int N, cudaStream_t stream) {
  const long long total = (long long)(K / 8) * (N / 8);
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  long long blocks = (total + threads - 1) / threads;
  const long long cap = 148LL * 16;  // enough resident work to saturate HBM
  if (blocks > cap) blocks = cap;
  if (out_bf16)
    dequant_kernel<true><<<(unsigned)blocks, threads, 0, stream>>>(
        packed, static_cast<const __half*>(scales), out, K, N);
  else
    dequant_kernel<false><<<(unsigned)blocks, threads, 0, stream>>>(
        packed, static_cast<const __half*>(scales), out, K, N);
  return cudaGetLastError();
}

}  // namespace w4
