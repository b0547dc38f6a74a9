/*
 * w4_oracle.c - C restatement of the reference's W4A16 path, for the CPU.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA library and the timed
 * CPU baseline (the reference's dequantise-then-matmul path on host cores).
 * The product never links or loads it. Built by oracle/build.py into
 * oracle/libw4oracle.so.
 *
 * Restated from raihan-js/roofline-decoding src/roofline/kernels.py:
 *   w4o_pack            kernels.py:24-47   (pack_weights)
 *   w4o_dequant_fp16    kernels.py:50-74   (_dequant_kernel: fp32 product, fp16 store)
 *   w4o_dequant_matmul  kernels.py:77-90 then kernels.py:271-273: materialise the
 *                       fp16 weight, then x.float() @ W.float() (the CPU path the
 *                       reference's tests and v1 use), OpenMP over columns
 *   w4o_gemv_exact      the v2/v3 sum (kernels.py:93-128) in double
 * fp16 conversions use the compiler's _Float16 (IEEE round-to-nearest-even).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline float h2f(uint16_t h) {
  _Float16 v;
  memcpy(&v, &h, 2);
  return (float)v;
}
static inline uint16_t f2h(float f) {
  _Float16 v = (_Float16)f;
  uint16_t h;
  memcpy(&h, &v, 2);
  return h;
}
static inline float bf2f(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

int w4o_version(void) { return 1; }

int w4o_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Sets the OpenMP thread count of the following parallel regions (a process
   launcher may have set OMP_NUM_THREADS=1); returns the new maximum. */
int w4o_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
  return omp_get_max_threads();
#else
  (void)n;
  return 1;
#endif
}

/* nan_as_cpu: 0 -> q = 0 where w/s is NaN (torch on a CUDA device),
 *             1 -> q = INT32_MIN (torch on x86), summed in int64 and wrapped. */
void w4o_pack(const uint16_t* w, int K, int N, int group_size, int nan_as_cpu,
              int32_t* packed, uint16_t* scales) {
  const int G = K / group_size;
#pragma omp parallel for schedule(static)
  for (long long gn = 0; gn < (long long)G * N; ++gn) {
    const int grp = (int)(gn / N), n = (int)(gn % N);
    float amax = 0.f;
    int has_nan = 0;
    for (int r = 0; r < group_size; ++r) {
      const float v = h2f(w[(size_t)(grp * group_size + r) * N + n]);
      if (isnan(v)) has_nan = 1;
      const float a = fabsf(v);
      if (a > amax) amax = a;
    }
    if (has_nan) amax = NAN;
    else if (amax < 1e-8f) amax = 1e-8f;
    const uint16_t sh = f2h(amax / 7.0f);
    scales[(size_t)grp * N + n] = sh;
    const float s = h2f(sh);
    for (int j = 0; j < group_size / 8; ++j) {
      int64_t sum = 0;
      for (int i = 0; i < 8; ++i) {
        const float v = h2f(w[(size_t)(grp * group_size + 8 * j + i) * N + n]);
        float q = rintf(v / s) + 8.0f;
        int64_t qi;
        if (isnan(q)) qi = nan_as_cpu ? (int64_t)INT32_MIN : 0;
        else qi = (int64_t)(q < 0.f ? 0.f : (q > 15.f ? 15.f : q));
        sum += (int64_t)((uint64_t)qi << (4 * i));
      }
      packed[(size_t)(grp * (group_size / 8) + j) * N + n] = (int32_t)(uint32_t)(uint64_t)sum;
    }
  }
}

static inline float deq(uint32_t word, int nib, float s) {
  return (float)((int)((word >> (4 * nib)) & 0xFu) - 8) * s;
}

void w4o_dequant_fp16(const int32_t* packed, const uint16_t* scales, int K, int N,
                      uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (int k8 = 0; k8 < K / 8; ++k8) {
    const int grp = k8 * 8 / 128;
    for (int n = 0; n < N; ++n) {
      const uint32_t word = (uint32_t)packed[(size_t)k8 * N + n];
      const float s = h2f(scales[(size_t)grp * N + n]);
      for (int i = 0; i < 8; ++i) out[(size_t)(k8 * 8 + i) * N + n] = f2h(deq(word, i, s));
    }
  }
}

/* y[M, N] (fp32) = x[M, K] @ fp16(dequant(W)). x is fp16 (x_bf16 = 0) or bf16
 * bit patterns. wbuf: caller scratch of K*N uint16 for the materialised
 * weight (the v1 pass). */
void w4o_dequant_matmul(const uint16_t* x, int x_bf16, int M, const int32_t* packed,
                        const uint16_t* scales, int K, int N, uint16_t* wbuf, float* y) {
  w4o_dequant_fp16(packed, scales, K, N, wbuf);
  const int NB = 256;
  const int nblocks = (N + NB - 1) / NB;
#pragma omp parallel for schedule(static)
  for (int b = 0; b < nblocks * M; ++b) {
    const int m = b / nblocks, n0 = (b % nblocks) * NB;
    const int n1 = n0 + NB < N ? n0 + NB : N;
    float acc[256];
    for (int n = n0; n < n1; ++n) acc[n - n0] = 0.f;
    for (int k = 0; k < K; ++k) {
      const uint16_t xb = x[(size_t)m * K + k];
      const float xv = x_bf16 ? bf2f(xb) : h2f(xb);
      const uint16_t* wr = wbuf + (size_t)k * N;
      for (int n = n0; n < n1; ++n) acc[n - n0] += xv * h2f(wr[n]);
    }
    for (int n = n0; n < n1; ++n) y[(size_t)m * N + n] = acc[n - n0];
  }
}

/* y[M, N] (double) = sum_k x (q - 8) s with fp32 weights, accumulated in double. */
void w4o_gemv_exact(const uint16_t* x, int x_bf16, int M, const int32_t* packed,
                    const uint16_t* scales, int K, int N, double* y) {
#pragma omp parallel for schedule(static)
  for (long long mn = 0; mn < (long long)M * N; ++mn) {
    const int m = (int)(mn / N), n = (int)(mn % N);
    double acc = 0.0;
    for (int k8 = 0; k8 < K / 8; ++k8) {
      const uint32_t word = (uint32_t)packed[(size_t)k8 * N + n];
      const float s = h2f(scales[(size_t)(k8 * 8 / 128) * N + n]);
      for (int i = 0; i < 8; ++i) {
        const uint16_t xb = x[(size_t)m * K + k8 * 8 + i];
        const double xv = x_bf16 ? bf2f(xb) : h2f(xb);
        acc += xv * (double)deq(word, i, s);
      }
    }
    y[mn] = acc;
  }
}
