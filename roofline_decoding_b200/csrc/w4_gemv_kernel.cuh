// w4_gemv_kernel.cuh - the fused W4A16 dequantise + GEMV / small-M GEMM kernel
// for sm_100a (device code; instantiated by w4_gemv.cu, w4_gemv_ops.cu and
// w4_gemv_fused.cu).
//
// Computes y[m, n] = sum_k x[m, k] * (q[k, n] - 8) * s[k / 128, n] for
// 1 <= M <= 16, the operation of roofline/kernels.py:93-128 (_fused_gemv_kernel)
// and :163-208 (_fused_gemv_v3_kernel), on the reference's packed layout.
//
// Work decomposition
//   CTA tile    : 32*SW output columns x one K slice (a "split"). With fewer
//                 CTA columns C than tiles T (large N), CTA column i takes
//                 the tiles i, i + C, i + 2C, ... and its producer streams
//                 them back to back through one ring; the x slice is staged
//                 once, and each tile's partial sums stay in shared memory
//                 until the common epilogue. These streaming instances also
//                 come with 16 compute warps (one CTA per SM) and stage bf16
//                 activations as fp16 (a cheaper unpack in the K loop).
//   Warps       : SW*RG compute warps + 1 producer warp. Compute warp w owns
//                 strip w % SW (32 columns) and row group w / SW.
//   Stage       : RG K-groups (RG * 16 packed rows) for all SW strips, i.e.
//                 SW TMA boxes of [RG*16 rows x 32 int32] (128B-swizzled) plus
//                 one box of RG x 32*SW fp16 scales. The producer streams
//                 stages through an mbarrier ring of `stages` slots.
//   Split-K     : the splits of one column tile form a thread-block cluster;
//                 after the K loop every CTA leaves its fp32 partial in shared
//                 memory and the cluster sums them over DSMEM in rank order.
//                 No atomics, no workspace: results are bit-reproducible.
//
// Inner product on the tensor cores (swap-AB): A = W^T tile (16 columns x 16
// k), B = x^T (16 k x 8 batch rows), D fp32. A thread's 16-byte shared load
// yields 4 columns x 8 k of one packed row; LOP3 turns each word into four
// f16x2/bf16x2 pairs of exact small integers, (q - 8) plus a constant that a
// per-(group, row) correction removes from the sum. The k order inside an MMA is a
// permutation of the true k order (nibbles (0,4),(1,5) | (2,6),(3,7) of the
// rows 2t, 2t+1 of each 8-row octet); x is staged in shared memory in the same
// permuted order, so the sum is unchanged. The per-group scale multiplies the
// fp32 group sum once per (group, column) - fused in registers.
#pragma once

#include "w4_internal.h"
#include "w4_ptx.cuh"

#include <cooperative_groups.h>

#include <algorithm>

namespace cg = cooperative_groups;

namespace w4 {

__device__ __forceinline__ float2 h2f2(uint32_t v, bool bf16) {
  if (bf16) return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v));
  return __half22float2(*reinterpret_cast<const __half2*>(&v));
}

struct GemvParams {
  const void* x;  // [M, K] fp16 / bf16
  void* y;        // [M, N] fp16 / bf16
  int M, K, N;
  int groups_total;      // K / 128
  int groups_per_split;  // K groups handled by one CTA
  int n_tiles;           // column tiles (32*SW columns each) covering N
  int tiles_per_cta;     // most tiles one CTA column takes (partial-sum space)
  int stages;            // ring depth
  int y_bf16;
  int* err;  // device error word
  // fused operations (decode step); all zero for a plain GEMV
  int pro;             // W4_PRO_*: transform applied to x while staging it
  const void* pro_w;   // RMSNorm weight [K] (x's type)
  float eps;           // RMSNorm epsilon
  int epi;             // W4_EPI_*: transform applied to y before the store
  const void* epi_src; // bias [N] or residual [M, N] (y's type; may alias y)
};

// Column-parallel output: this rank's slice of y goes to every rank's buffer
// of the current parity, then a flag per rank says the slice is complete.
struct PeerParams {
  int world;            // 0: a plain GEMV (the fields below are unused)
  int rank, n_full, col_off;
  void* y[2][W4B200_MAX_PEERS];
  unsigned* flags[W4B200_MAX_PEERS];  // rank q's flag words; word r is set by rank r
  unsigned* state;                    // [0] epoch of the last completed call, [1] CTAs done
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Operation sets a kernel instance is compiled for. A plain GEMV and each
// fused combination of the decode step get an instance that contains only
// their own prologue/epilogue code (a smaller kernel: in a chain of dependent
// launches its post-wait path is fetched faster), and so does the plain GEMV
// with the gathered (peer) output; any other combination, and a gathered
// output with a prologue, epilogue or several tiles per CTA, take the generic
// instance, which selects at run time.
enum : int {
  kOpsPlain = 0,           // no prologue, no epilogue, local output
  kOpsGeneric = 1,         // prologue, epilogue and peer output chosen at run time
  kOpsRmsBias = 2,         // RMSNorm prologue, bias epilogue (q|k|v)
  kOpsRms = 3,             // RMSNorm prologue (gate|up)
  kOpsResidual = 4,        // residual epilogue (o)
  kOpsSwigluResidual = 5,  // SwiGLU prologue, residual epilogue (down)
  kOpsRmsSwiglu = 6,       // RMSNorm prologue, SwiGLU epilogue (gate|up, interleaved)
  kOpsPlainTiles = 7,      // plain, CTA columns streaming several column tiles
  kOpsPeer = 8,            // plain, output gathered into every rank's buffer
};
constexpr int kOpsFusedFirst = kOpsRmsBias, kOpsFusedLast = kOpsRmsSwiglu;
// Instances whose CTA columns may take several column tiles (the others are
// compiled for one tile per CTA: the loop over tiles costs registers).
constexpr bool ops_tiles(int ops) { return ops == kOpsGeneric || ops == kOpsPlainTiles; }
constexpr int ops_pro(int ops) {
  return (ops == kOpsRmsBias || ops == kOpsRms || ops == kOpsRmsSwiglu) ? W4_PRO_RMSNORM
         : ops == kOpsSwigluResidual            ? W4_PRO_SWIGLU
                                                : W4_PRO_NONE;
}
constexpr int ops_epi(int ops) {
  return ops == kOpsRmsBias                                     ? W4_EPI_BIAS
         : (ops == kOpsResidual || ops == kOpsSwigluResidual) ? W4_EPI_RESIDUAL
         : ops == kOpsRmsSwiglu                                 ? W4_EPI_SWIGLU
                                                               : W4_EPI_NONE;
}
// The fused instance for a (prologue, epilogue) pair, or kOpsGeneric.
constexpr int ops_for(int pro, int epi) {
  return (pro == W4_PRO_NONE && epi == W4_EPI_NONE)         ? kOpsPlain
         : (pro == W4_PRO_RMSNORM && epi == W4_EPI_BIAS)    ? kOpsRmsBias
         : (pro == W4_PRO_RMSNORM && epi == W4_EPI_NONE)    ? kOpsRms
         : (pro == W4_PRO_NONE && epi == W4_EPI_RESIDUAL)   ? kOpsResidual
         : (pro == W4_PRO_SWIGLU && epi == W4_EPI_RESIDUAL) ? kOpsSwigluResidual
         : (pro == W4_PRO_RMSNORM && epi == W4_EPI_SWIGLU)  ? kOpsRmsSwiglu
                                                            : kOpsGeneric;
}

constexpr int kErrPeerWait = 6;    // a peer's completion flag did not arrive in time


__device__ __forceinline__ float ld_f(const void* p, size_t i, bool bf16) {
  const uint16_t v = static_cast<const uint16_t*>(p)[i];
  return bf16 ? __uint_as_float((uint32_t)v << 16) : __half2float(__ushort_as_half(v));
}
__device__ __forceinline__ float round_to(float v, bool bf16) {
  return bf16 ? __bfloat162float(__float2bfloat16_rn(v)) : __half2float(__float2half_rn(v));
}
__device__ __forceinline__ uint32_t pack2(float a, float b, bool bf16) {
  if (bf16) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
  const __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Applies the staging transform to 8 consecutive activations x[m, k..k+7]
// (aux holds the matching 8 values of the second operand, loaded by the
// caller in the same batch as x):
//   RMSNorm: round(round(x * inv_rms) * w[k])   aux = w[k..k+7] (Qwen2/Llama
//            RMSNorm: fp32 normalisation, cast to the activation type, times
//            the weight)
//   SwiGLU : round(round(silu(g)) * u)           x = gate, aux = up (silu in
//            fp32, cast; product cast)
template <bool kBF16>
__device__ __forceinline__ uint4 stage_transform(int pro, uint4 v, uint4 aux, float inv_rms) {
  const uint32_t* xi = reinterpret_cast<const uint32_t*>(&v);
  const uint32_t* ai = reinterpret_cast<const uint32_t*>(&aux);
  uint4 o;
  uint32_t* oi = reinterpret_cast<uint32_t*>(&o);
  if (pro == W4_PRO_RMSNORM) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 xf = h2f2(xi[i], kBF16), wf = h2f2(ai[i], kBF16);
      oi[i] = pack2(round_to(xf.x * inv_rms, kBF16) * wf.x,
                    round_to(xf.y * inv_rms, kBF16) * wf.y, kBF16);
    }
    return o;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 g = h2f2(xi[i], kBF16), u = h2f2(ai[i], kBF16);
    const float sa = round_to(g.x / (1.0f + __expf(-g.x)), kBF16);
    const float sb = round_to(g.y / (1.0f + __expf(-g.y)), kBF16);
    oi[i] = pack2(sa * u.x, sb * u.y, kBF16);
  }
  return o;
}

template <int SW, int RG>
struct TileShape {
  static constexpr int kCW = SW * RG;              // compute warps
  static constexpr int kThreads = (kCW + 1) * 32;  // + producer warp
  static constexpr int kNT = 32 * SW;              // output columns per CTA
  static constexpr int kStripBytes = RG * 16 * 128;
  static constexpr int kStageBytes = SW * kStripBytes;
  static constexpr int kScaleBytes = RG * kNT * 2;                // one scale box
  static constexpr int kScaleSlot = (kScaleBytes + 127) / 128 * 128;  // TMA dst: 128 B aligned
};

__device__ __forceinline__ void consumer_bar_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

__device__ __forceinline__ void report_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// Reorders the 8 activations of one packed row into the order the MMA
// fragments consume them: (x0,x4) (x1,x5) (x2,x6) (x3,x7). In fp16 the odd
// pairs meet the "1024 + 16q" form of unpack_nibbles and are pre-scaled by
// 1/16 (exact for normal values; below 2^-10 the rounding error is under
// 2^-25 absolute).
template <bool kBF16Math>
__device__ __forceinline__ uint4 permute_row(uint4 v) {
  uint4 o;
  o.x = __byte_perm(v.x, v.z, 0x5410);
  o.y = __byte_perm(v.x, v.z, 0x7632);
  o.z = __byte_perm(v.y, v.w, 0x5410);
  o.w = __byte_perm(v.y, v.w, 0x7632);
  if constexpr (!kBF16Math) {
    constexpr uint32_t kSixteenth = 0x2C002C00u;  // 1/16 | 1/16
    constexpr uint32_t kZero = 0x80008000u;       // -0 | -0 (keeps x * 1/16 exact)
    o.y = fma_f16x2(o.y, kSixteenth, kZero);
    o.w = fma_f16x2(o.w, kSixteenth, kZero);
  }
  return o;
}

// 8 bf16 activations of one packed row -> fp16, times the power of two 2^e
// of their K group: 16 consecutive lanes hold the 16 rows of a group (every
// lane of the warp calls this; lanes past the data pass zeros). The lane
// with `leader` set stores the group's 2^-e to *pow_out.
__device__ __forceinline__ uint4 bf16_row_to_f16(uint4 v, bool leader, float* pow_out) {
  const uint32_t* vi = reinterpret_cast<const uint32_t*>(&v);
  float f[8];
  float mx = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(vi[i] << 16);
    f[2 * i + 1] = __uint_as_float(vi[i] & 0xFFFF0000u);
    mx = fmaxf(mx, fmaxf(fabsf(f[2 * i]), fabsf(f[2 * i + 1])));
  }
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  // biased exponent eb of mx: mx * 2^(141 - eb) lies in [2^14, 2^15)
  const int eb = (int)((__float_as_uint(mx) >> 23) & 0xFFu);
  const int e = mx > 0.f ? min(126, max(-126, 141 - eb)) : 0;
  const float up = __uint_as_float((uint32_t)(127 + e) << 23);
  if (leader) *pow_out = __uint_as_float((uint32_t)(127 - e) << 23);
  uint4 o;
  uint32_t* oi = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 h = __floats2half2_rn(f[2 * i] * up, f[2 * i + 1] * up);
    oi[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return o;
}


// Stages the activations of K groups [g0, g1) of every batch row in shared
// memory, in the order the MMA fragments consume them (permute_row), with the
// prologue applied; leaves beta[m][group] (the unpack constant summed against
// the group's activations) and, for RMSNorm, 1/rms per row. Run by the kCW
// compute warps only; ends with a barrier among them.
// Packed row of activation element group idx of a staging pass (8 activations
// of batch row m); false past the slice.
__device__ __forceinline__ bool stage_row(int idx, int total, int rows_slice, int g0, int g1,
                                          int* m, int* krow) {
  if (idx >= total) return false;
  *m = idx / rows_slice;
  *krow = g0 * 16 + (idx - *m * rows_slice);
  return *krow < g1 * 16;
}

// The RMSNorm weights of this thread's first staged row: they do not depend
// on the previous kernel, so they are loaded before the grid-dependency wait
// (a per-layer constant is rarely still in L2). Later rows load as they stage.
__device__ __forceinline__ uint4 preload_norm_weight(const GemvParams& p, int g0, int g1, int gps) {
  const int rows_slice = gps * 16;
  int m, krow;
  if (stage_row((int)threadIdx.x, p.M * rows_slice, rows_slice, g0, g1, &m, &krow))
    return __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.pro_w) +
                                                (size_t)krow * 8));
  return make_uint4(0u, 0u, 0u, 0u);
}

// kF16Math: bf16 rows are converted to fp16 for the MMAs (below).
template <bool kBF16, int kCW, bool kF16Math>
__device__ __forceinline__ void stage_activations(const GemvParams& p, int g0, int g1, int gps,
                                                  uint8_t* s_x, int plane, float* s_beta,
                                                  float* s_pow, float* s_inv, float* s_red,
                                                  int warp, int lane, uint4 pre, int pro) {
  constexpr int nct = kCW * 32;
  const int M = p.M;
  const int rows_slice = gps * 16;
  const uint16_t* xg = static_cast<const uint16_t*>(p.x);
  // x row pitch: a SwiGLU prologue reads gate|up rows of 2K
  const size_t x_pitch = (pro == W4_PRO_SWIGLU) ? 2 * (size_t)p.K : (size_t)p.K;
  // RMSNorm needs 1/rms of the whole row. When this CTA stages the whole row
  // of a single activation row in one batch (the decode case), the sum of
  // squares comes from the staging loads themselves (one global round
  // trip); otherwise a pre-pass over the row computes it first.
  const bool rms_one_pass = pro == W4_PRO_RMSNORM && M == 1 && g0 == 0 &&
                            g1 == p.groups_total && rows_slice <= 4 * nct;
  if (pro == W4_PRO_RMSNORM && !rms_one_pass) {
    // inv_rms[m] over the whole row (every CTA recomputes it: K <= 28672
    // activations, served from L2), reduced in a fixed order
    float* s_part = s_red;  // scratch: [kCW][M] partial sums (s_red is free until the epilogue)
    for (int m = 0; m < M; ++m) {
      float acc2 = 0.f;
      for (int i = threadIdx.x; i < p.K / 8; i += nct) {
        const uint4 v = __ldcg(reinterpret_cast<const uint4*>(xg + m * x_pitch + 8 * (size_t)i));
        const uint32_t* vi = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = h2f2(vi[e], kBF16);
          acc2 = fmaf(f.x, f.x, acc2);
          acc2 = fmaf(f.y, f.y, acc2);
        }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) acc2 += __shfl_xor_sync(0xffffffffu, acc2, off);
      if (lane == 0) s_part[warp * M + m] = acc2;
    }
    consumer_bar_sync(nct);
    if (threadIdx.x < M) {
      float tot = 0.f;
      for (int w = 0; w < kCW; ++w) tot += s_part[w * M + threadIdx.x];
      s_inv[threadIdx.x] = rsqrtf(tot / (float)p.K + p.eps);
    }
    consumer_bar_sync(nct);
  }
  // Batches of 4 independent 16-byte loads per thread, all in flight before
  // the first is consumed (one global round trip per batch, not per row).
  // 16 consecutive threads hold the 16 rows of one group, so the group's
  // correction beta is a 16-lane shuffle reduction (nct and rows_slice are
  // multiples of 16, so a 16-lane group never straddles two groups).
  const int total = M * rows_slice;
  // b0 is the same for every consumer thread, so all of them run the same
  // trips and every shuffle below has its full warp
  float inv_one = 0.f;  // 1/rms of the single row when it is summed in one pass
  for (int b0 = 0; b0 < total; b0 += 4 * nct) {
    uint4 v[4], aux[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int idx = b0 + u * nct + threadIdx.x;
      v[u] = make_uint4(0u, 0u, 0u, 0u);
      aux[u] = make_uint4(0u, 0u, 0u, 0u);
      if (idx < total) {
        const int m = idx / rows_slice;
        const int krow = g0 * 16 + (idx - m * rows_slice);  // packed row = 8 activations
        if (krow < g1 * 16) {
          const uint16_t* xr = xg + (size_t)m * x_pitch + (size_t)krow * 8;
          v[u] = __ldcg(reinterpret_cast<const uint4*>(xr));
          if (pro == W4_PRO_RMSNORM)
            aux[u] = (b0 == 0 && u == 0)
                         ? pre
                         : __ldg(reinterpret_cast<const uint4*>(
                               static_cast<const uint16_t*>(p.pro_w) + (size_t)krow * 8));
          else if (pro == W4_PRO_SWIGLU)
            aux[u] = __ldcg(reinterpret_cast<const uint4*>(xr + p.K));
        }
      }
    }
    if (rms_one_pass) {  // sum of squares of the (whole, single) row from registers
      float acc2 = 0.f;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t* vi = reinterpret_cast<const uint32_t*>(&v[u]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = h2f2(vi[e], kBF16);
          acc2 = fmaf(f.x, f.x, acc2);
          acc2 = fmaf(f.y, f.y, acc2);
        }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) acc2 += __shfl_xor_sync(0xffffffffu, acc2, off);
      if (lane == 0) s_red[warp] = acc2;
      consumer_bar_sync(nct);
      // every thread sums the warps' parts itself, in the same order: one
      // barrier instead of a second barrier after a single thread's sum
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < kCW; ++w) tot += s_red[w];
      inv_one = rsqrtf(tot / (float)p.K + p.eps);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (b0 + u * nct >= total) break;  // uniform over the consumer threads
      const int idx = b0 + u * nct + threadIdx.x;
      float lo = 0.f, hi = 0.f;
      int m = 0, r = 0;
      if (idx < total) {
        m = idx / rows_slice;
        r = idx - m * rows_slice;
        if (pro != W4_PRO_NONE && g0 * 16 + r < g1 * 16)
          v[u] = stage_transform<kBF16>(
              pro, v[u], aux[u],
              pro == W4_PRO_RMSNORM ? (rms_one_pass ? inv_one : s_inv[m]) : 0.f);
      }
      // With kF16Math, bf16 rows enter the MMAs as fp16 (whose unpack costs 5
      // operations per packed word against 7): every group is scaled by the
      // power of two 2^e that puts its largest |x| in [2^14, 2^15), so the
      // conversion is exact (8 significant bits into 11) for every element
      // within 2^-28 of the group's largest; the group's sum is scaled back
      // by 2^-e, also exact.
      constexpr bool kBF16Math = kBF16 && !kF16Math;
      if constexpr (kBF16 && kF16Math)
        v[u] = bf16_row_to_f16(v[u], idx < total && (idx & 15) == 0, s_pow + (idx >> 4));
      if (idx < total) {
        const uint4 o = permute_row<kBF16Math>(v[u]);
        *reinterpret_cast<uint4*>(s_x + m * plane + r * 16) = o;
        const float2 a = h2f2(o.x, kBF16Math), b = h2f2(o.y, kBF16Math);
        const float2 c = h2f2(o.z, kBF16Math), d = h2f2(o.w, kBF16Math);
        lo = (a.x + a.y) + (c.x + c.y);
        hi = (b.x + b.y) + (d.x + d.y);
      }
      float bsum = kBF16Math ? kBF16Offset * (lo + hi) : kF16LowOffset * lo + kF16HighOffset * hi;
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) bsum += __shfl_xor_sync(0xffffffffu, bsum, off);
      if (idx < total && (idx & 15) == 0) s_beta[idx >> 4] = bsum;
    }
  }
  consumer_bar_sync(nct);
}

// Shared-memory addresses one compute lane reads in every stage:
//   weights: rows rg*16 + 8*o + 2t + e of its strip's box, 16-byte chunk g
//            stored at chunk g ^ (row & 7) by the 128B swizzle;
//   x:       lanes whose batch row g >= M read row M-1 instead, so every
//            lane loads unconditionally (their output columns are unused);
//   beta:    likewise clamped.
template <int MB, int SW, int RG>
struct LaneView {
  uint32_t w_off[2];
  uint32_t x_off[MB];
  const float* b_row[MB][2];
  int pow_off;  // s_pow - s_beta, in floats (bf16 activations: 2^-e per group)
  uint32_t sc_off;

  __device__ __forceinline__ LaneView(const uint8_t* s_w, const uint8_t* s_x, const uint8_t* s_sc,
                                      const float* s_beta, int pow_off, int plane, int gps, int M,
                                      int strip, int rg, int g, int t)
      : pow_off(pow_off) {
    using T = TileShape<SW, RG>;
#pragma unroll
    for (int e = 0; e < 2; ++e)
      w_off[e] = smem_u32(s_w) + strip * T::kStripBytes + (rg * 16 + 2 * t + e) * 128 +
                 ((g ^ (2 * t + e)) << 4);
#pragma unroll
    for (int mb = 0; mb < MB; ++mb) {
      x_off[mb] = smem_u32(s_x) + min(8 * mb + g, M - 1) * plane + 2 * t * 16;
      b_row[mb][0] = s_beta + min(8 * mb + 2 * t, M - 1) * gps;
      b_row[mb][1] = s_beta + min(8 * mb + 2 * t + 1, M - 1) * gps;
    }
    sc_off = smem_u32(s_sc) + (rg * T::kNT + 32 * strip + 4 * g) * 2;
  }
};

// One K group of one stage for one compute warp: acc += s * sum_k (q - 8) x
// over the group gl of the staged activations, its weights in the ring slot
// at byte offset stage_base and its scales in the scale slot at sc.
// kBF16Math: bf16 MMAs on bf16 activations; otherwise fp16 MMAs, on fp16
// activations or bf16 ones converted with a power of two per group (kPow).
template <bool kBF16Math, bool kPow, int MB, int SW, int RG>
__device__ __forceinline__ void mma_group(float (&acc)[2][MB][4], const LaneView<MB, SW, RG>& lv,
                                          uint32_t stage_base, uint32_t sc, int gl) {
  // accumulators start at -beta of their batch row: the MMA sums then
  // leave exactly sum_k (q - 8) x of this group
  float c[2][MB][4];
#pragma unroll
  for (int mb = 0; mb < MB; ++mb) {
    const float nb0 = -lv.b_row[mb][0][gl];
    const float nb1 = -lv.b_row[mb][1][gl];
#pragma unroll
    for (int a = 0; a < 2; ++a) {
      c[a][mb][0] = nb0;
      c[a][mb][1] = nb1;
      c[a][mb][2] = nb0;
      c[a][mb][3] = nb1;
    }
  }
#pragma unroll
  for (int o = 0; o < 2; ++o) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const uint4 wv = lds128(lv.w_off[e] + stage_base + o * 1024);
      const uint32_t xrow = (gl * 16 + 8 * o + e) * 16;
      uint4 xb[MB];
#pragma unroll
      for (int mb = 0; mb < MB; ++mb) xb[mb] = lds128(lv.x_off[mb] + xrow);
      uint32_t ha[4], hb[4];
      unpack_nibbles<kBF16Math>(wv.x, ha);  // column 4g
      unpack_nibbles<kBF16Math>(wv.y, hb);  // column 4g+1
#pragma unroll
      for (int mb = 0; mb < MB; ++mb) {
        mma_16816<kBF16Math>(c[0][mb], ha[0], hb[0], ha[1], hb[1], xb[mb].x, xb[mb].y);
        mma_16816<kBF16Math>(c[0][mb], ha[2], hb[2], ha[3], hb[3], xb[mb].z, xb[mb].w);
      }
      unpack_nibbles<kBF16Math>(wv.z, ha);  // column 4g+2
      unpack_nibbles<kBF16Math>(wv.w, hb);  // column 4g+3
#pragma unroll
      for (int mb = 0; mb < MB; ++mb) {
        mma_16816<kBF16Math>(c[1][mb], ha[0], hb[0], ha[1], hb[1], xb[mb].x, xb[mb].y);
        mma_16816<kBF16Math>(c[1][mb], ha[2], hb[2], ha[3], hb[3], xb[mb].z, xb[mb].w);
      }
    }
  }
  // Scales of this group for columns (4g, 4g+1) and (4g+2, 4g+3).
  const uint32_t s01 = lds32(sc);
  const uint32_t s23 = lds32(sc + 4);
  const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&s01));
  const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&s23));
#pragma unroll
  for (int mb = 0; mb < MB; ++mb) {
    // bf16 activations: the group's 2^-e of batch rows 2t (i even), 2t+1 (i odd)
    const float p0 = kPow ? lv.b_row[mb][0][gl + lv.pow_off] : 1.f;
    const float p1 = kPow ? lv.b_row[mb][1][gl + lv.pow_off] : 1.f;
    acc[0][mb][0] = fmaf(f01.x * p0, c[0][mb][0], acc[0][mb][0]);
    acc[0][mb][1] = fmaf(f01.x * p1, c[0][mb][1], acc[0][mb][1]);
    acc[0][mb][2] = fmaf(f01.y * p0, c[0][mb][2], acc[0][mb][2]);
    acc[0][mb][3] = fmaf(f01.y * p1, c[0][mb][3], acc[0][mb][3]);
    acc[1][mb][0] = fmaf(f23.x * p0, c[1][mb][0], acc[1][mb][0]);
    acc[1][mb][1] = fmaf(f23.x * p1, c[1][mb][1], acc[1][mb][1]);
    acc[1][mb][2] = fmaf(f23.y * p0, c[1][mb][2], acc[1][mb][2]);
    acc[1][mb][3] = fmaf(f23.y * p1, c[1][mb][3], acc[1][mb][3]);
  }
}

// A compute warp's accumulators into s_red[rg][m][col] (rows m < M only).
template <int MB, int NT>
__device__ __forceinline__ void write_partials(const float (&acc)[2][MB][4], float* s_red, int M,
                                               int strip, int rg, int g, int t) {
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int mb = 0; mb < MB; ++mb)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int m = 8 * mb + 2 * t + (i & 1);
        if (m < M) {
          const int col = 32 * strip + 4 * g + 2 * a + (i >> 1);
          s_red[(rg * M + m) * NT + col] = acc[a][mb][i];
        }
      }
}

// Writes y[m, n] = v with the epilogue applied (n < N): to y, or for a
// gathered output to every rank's buffer of this call's parity.
// e is the epilogue's operand of this element (bias[n] or residual[m, n],
// already loaded into shared memory; unused without an epilogue).
__device__ __forceinline__ void store_out(const GemvParams& p, const PeerParams& pp, int epi,
                                          int world, unsigned epoch, int m, int n, float v,
                                          float e) {
  if (n >= p.N) return;
  if (epi == W4_EPI_BIAS) {
    v += e;  // one rounding, like a GEMM's bias epilogue
  } else if (epi == W4_EPI_RESIDUAL) {
    // out = round(residual + round(y)): the layer output is rounded before
    // the residual add, as in the reference model's bf16 forward
    v = e + round_to(v, p.y_bf16);
  }
  if (world > 0) {  // every rank's buffer of this parity (NVLink stores)
    const size_t at = (size_t)m * pp.n_full + pp.col_off + n;
    const int par = (int)(epoch & 1u);
    for (int q = 0; q < pp.world; ++q) {
      if (p.y_bf16)
        static_cast<__nv_bfloat16*>(pp.y[par][q])[at] = __float2bfloat16_rn(v);
      else
        static_cast<__half*>(pp.y[par][q])[at] = __float2half_rn(v);
    }
  } else if (p.y_bf16) {
    static_cast<__nv_bfloat16*>(p.y)[(size_t)m * p.N + n] = __float2bfloat16_rn(v);
  } else {
    static_cast<__half*>(p.y)[(size_t)m * p.N + n] = __float2half_rn(v);
  }
}

// Gathered output: the CTA that finishes last on this rank publishes the
// epoch to every rank, then waits until every rank published it here. Each
// CTA orders its peer stores before its count at GPU scope (a cumulative
// release); the last CTA, having observed every count, makes all of them
// visible system-wide with one system-scope fence before it publishes. Call
// after a __syncthreads that follows the CTA's last store.
__device__ __forceinline__ void publish_gathered(const GemvParams& p, const PeerParams& pp,
                                                 unsigned epoch, unsigned ctas) {
  if (threadIdx.x != 0) return;
  __threadfence();
  if (atomicAdd(&pp.state[1], 1u) == ctas - 1) {
    __threadfence_system();
    for (int q = 0; q < pp.world; ++q) st_release_sys(pp.flags[q] + pp.rank, epoch);
    const unsigned* mine = pp.flags[pp.rank];
    for (int q = 0; q < pp.world; ++q) {
      const unsigned long long t0 = globaltimer_ns();
      while ((int)(ld_acquire_sys(mine + q) - epoch) < 0) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          report_error(p.err, kErrPeerWait);
          break;
        }
      }
    }
    pp.state[1] = 0u;
    pp.state[0] = epoch;
    __threadfence();
  }
}

// Two CTAs per SM bound the registers (about 113 for 288 threads). The down
// projection's SwiGLU instance runs as a split-K grid of 2.6 CTAs per SM, so
// it is held to three (72 registers): a grid that does not fit the SMs at
// once runs in two waves.
// The 16-warp tiles (one CTA per SM, streaming) get the registers of one.
template <int OPS, int THREADS>
constexpr int gemv_min_blocks() {
  return THREADS > 288 ? 1 : OPS == kOpsSwigluResidual ? 3 : 2;
}

template <bool kBF16, int MB, int SW, int RG, int OPS>
__global__ void __launch_bounds__(TileShape<SW, RG>::kThreads,
                                  gemv_min_blocks<OPS, TileShape<SW, RG>::kThreads>())
    w4_gemv_kernel(const __grid_constant__ CUtensorMap tm_w,
                   const __grid_constant__ CUtensorMap tm_s, const GemvParams p,
                   const __grid_constant__ PeerParams pp) {
  using T = TileShape<SW, RG>;
  // the instance's operations: compile-time constants except in the generic one
  const int pro = OPS == kOpsGeneric ? p.pro : ops_pro(OPS);
  const int epi = OPS == kOpsGeneric ? p.epi : ops_epi(OPS);
  const int world = (OPS == kOpsGeneric || OPS == kOpsPeer) ? pp.world : 0;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  const int S = p.stages;
  const int M = p.M;
  const int gps = p.groups_per_split;
  const int plane = gps * 16 * 16 + 16;  // +16 B: odd batch rows land on other banks
  const int tile_elems = M * T::kNT;
  const int nsplit = gridDim.y;
  // this CTA column's tiles (one per CTA unless the grid has fewer columns)
  constexpr bool kTiles = ops_tiles(OPS);
  // bf16 activations: the streaming instances convert them to fp16 while
  // staging (a cheaper unpack in the throughput-bound K loop); the others,
  // run in chains of dependent launches, keep bf16 MMAs and the shorter
  // staging path.
  constexpr bool kF16Math = !kBF16 || OPS == kOpsPlainTiles;
  // CTA column c takes the tiles c, c + C, c + 2C, ... (C = gridDim.x), so
  // the CTAs running at once stream neighbouring columns (whole DRAM rows)
  const int t_first = (int)blockIdx.x;
  const int t_step = kTiles ? (int)gridDim.x : 1;
  const int n_tl = kTiles ? (p.n_tiles - t_first + t_step - 1) / t_step : 1;
  uint8_t* s_w = smem;
  uint8_t* s_sc = s_w + S * T::kStageBytes;
  uint8_t* s_x = s_sc + S * T::kScaleSlot;
  // beta[m][group]: the constant the unpacked values carry, summed against the
  // staged activations of each group (subtracted through the accumulator init)
  float* s_beta = reinterpret_cast<float*>(s_x + M * plane);
  const int n_beta = (M * gps + 3) & ~3;
  float* s_pow = s_beta + n_beta;  // bf16 activations: 2^-e per (row, group)
  float* s_inv = s_pow + n_beta;   // RMSNorm 1/rms per row
  float* s_red = s_inv + 16;
  float* s_epi = s_red + p.tiles_per_cta * RG * tile_elems;  // epilogue operand per element
  uint64_t* full = reinterpret_cast<uint64_t*>(s_epi + tile_elems);
  uint64_t* empty = full + S;
  unsigned& s_epoch = *reinterpret_cast<unsigned*>(empty + S);  // gathered output: this call's epoch

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = t_first * T::kNT;  // first column (the single-tile epilogues use it)
  const int g0 = blockIdx.y * gps;
  const int g1 = min(p.groups_total, g0 + gps);
  const int n_groups = max(0, g1 - g0);
  const int n_stages = (n_groups + RG - 1) / RG;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], T::kCW);
    }
    fence_mbar_init();
  }
  if (warp == T::kCW && lane == 0) {
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_s);
  }
  __syncthreads();
  // Every thread signals at once: the next grid of a PDL chain is scheduled as
  // soon as there is room on the SMs (shared memory bounds the overlap to about
  // two grids per SM), streams its weights while this one runs, and reads our
  // output only after its own grid-dependency wait.
  grid_launch_dependents();

  if (warp == T::kCW) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int issued = 0;
      int slot = 0;
      uint32_t phase = 0;  // phase of the current pass over the ring
      bool ok = true;
      for (int tl = 0; tl < n_tl && ok; ++tl) {
        const int c0 = (t_first + tl * t_step) * T::kNT;
        for (int j = 0; j < n_stages; ++j) {
          if (issued >= S && !mbar_wait(&empty[slot], phase ^ 1u)) {
            report_error(p.err, kErrEmptyWait);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[slot], T::kStageBytes + T::kScaleBytes);
          const int grp = g0 + j * RG;
#pragma unroll
          for (int s = 0; s < SW; ++s)
            tma_load_2d(s_w + slot * T::kStageBytes + s * T::kStripBytes, &tm_w, &full[slot],
                        c0 + 32 * s, grp * 16);
          tma_load_2d(s_sc + slot * T::kScaleSlot, &tm_s, &full[slot], c0, grp);
          ++issued;
          if (++slot == S) {
            slot = 0;
            phase ^= 1u;
          }
        }
      }
      // Do not leave while copies into this CTA's shared memory are in flight.
      for (int j = max(0, issued - S); j < issued; ++j)
        if (!mbar_wait(&full[j % S], (j / S) & 1)) report_error(p.err, kErrDrainWait);
    }

  } else {
    // ------------------------------------------------------------ consumers
    // Constants of the prologue and the epilogue (RMSNorm weight, bias) do not
    // depend on the previous kernel: load them before its completion.
    const uint4 pre = pro == W4_PRO_RMSNORM ? preload_norm_weight(p, g0, g1, gps)
                                              : make_uint4(0u, 0u, 0u, 0u);
    if (epi == W4_EPI_BIAS)
      for (int i = threadIdx.x; i < tile_elems; i += T::kCW * 32) {
        const int n = n0 + i % T::kNT;
        s_epi[i] = n < p.N ? ld_f(p.epi_src, n, p.y_bf16) : 0.f;
      }
    // x is produced by the previous kernel on the stream: wait for it.
    grid_dependency_wait();
    // the previous call's last CTA advanced the epoch before that grid ended
    if (world > 0 && threadIdx.x == 0) s_epoch = __ldcg(pp.state) + 1u;
    // The residual was written before x: its loads go out together with the
    // staging loads and land in shared memory before the epilogue.
    constexpr int kResPerThread = (8 * MB * T::kNT + T::kCW * 32 - 1) / (T::kCW * 32);
    float res[kResPerThread];
    const bool residual = epi == W4_EPI_RESIDUAL;
    if (residual) {
#pragma unroll
      for (int r = 0; r < kResPerThread; ++r) {
        const int i = threadIdx.x + r * T::kCW * 32;
        const int n = n0 + i % T::kNT;
        res[r] = (i < tile_elems && n < p.N)
                     ? ld_f(p.epi_src, (size_t)(i / T::kNT) * p.N + n, p.y_bf16)
                     : 0.f;
      }
    }
    stage_activations<kBF16, T::kCW, kF16Math>(p, g0, g1, gps, s_x, plane, s_beta, s_pow, s_inv, s_red,
                                     warp, lane, pre, pro);
    if (residual) {
#pragma unroll
      for (int r = 0; r < kResPerThread; ++r) {
        const int i = threadIdx.x + r * T::kCW * 32;
        if (i < tile_elems) s_epi[i] = res[r];
      }
    }

    const int strip = warp % SW;
    const int rg = warp / SW;
    const int g = lane >> 2;
    const int t = lane & 3;
    const LaneView<MB, SW, RG> lv(s_w, s_x, s_sc, s_beta, n_beta, plane, gps, M, strip, rg, g, t);

    int slot = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int tl = 0; tl < n_tl && ok; ++tl) {
      // acc[a][mb][i]: MMA tile a covers columns 4g+2a (i = 0,1) and 4g+2a+1
      // (i = 2,3); i & 1 selects batch row 8*mb + 2*(lane&3) + (i&1).
      float acc[2][MB][4];
#pragma unroll
      for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int b = 0; b < MB; ++b)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[a][b][i] = 0.f;

      for (int j = 0; j < n_stages; ++j) {
        if (!mbar_wait(&full[slot], phase)) {
          report_error(p.err, kErrFullWait);
          ok = false;
          break;
        }
        const int gl = j * RG + rg;  // group inside the slice
        if (gl < n_groups)
          mma_group<kBF16 && !kF16Math, kBF16 && kF16Math, MB, SW, RG>(acc, lv, slot * T::kStageBytes,
                                       lv.sc_off + slot * T::kScaleSlot, gl);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (++slot == S) {
          slot = 0;
          phase ^= 1u;
        }
      }
      write_partials<MB, T::kNT>(acc, s_red + tl * RG * tile_elems, M, strip, rg, g, t);
    }
  }
  __syncthreads();

  // Row groups -> plane 0, in a fixed order.
  if (epi == W4_EPI_SWIGLU) {
    // The tile's first half holds gate columns, its second half the matching
    // up columns (the weights alternate blocks of half a tile, 16 * SW); y
    // has half the columns. The bf16 arithmetic of the reference model's MLP:
    // gate and up rounded, silu in fp32 rounded, the product rounded by the
    // store. Host-checked: no split.
    constexpr int kHalf = T::kNT / 2;
    for (int o = threadIdx.x; o < M * kHalf; o += T::kThreads) {
      const int m = o / kHalf, c = o - m * kHalf;
      float gv = s_red[m * T::kNT + c], uv = s_red[m * T::kNT + kHalf + c];
#pragma unroll
      for (int r = 1; r < RG; ++r) {
        gv += s_red[(r * M + m) * T::kNT + c];
        uv += s_red[(r * M + m) * T::kNT + kHalf + c];
      }
      const int n = n0 / 2 + c;
      if (2 * n < p.N) {
        const float gr = round_to(gv, p.y_bf16), ur = round_to(uv, p.y_bf16);
        const float a = round_to(gr / (1.0f + __expf(-gr)), p.y_bf16);
        const size_t at = (size_t)m * (p.N / 2) + n;
        if (p.y_bf16)
          static_cast<__nv_bfloat16*>(p.y)[at] = __float2bfloat16_rn(a * ur);
        else
          static_cast<__half*>(p.y)[at] = __float2half_rn(a * ur);
      }
    }
  } else if (nsplit == 1) {
    // each thread sums its elements' row groups and stores them itself
    // (element i of the CTA's tiles: tile i / tile_elems, at i % tile_elems)
    const unsigned epoch = s_epoch;
    for (int idx = threadIdx.x; idx < n_tl * tile_elems; idx += T::kThreads) {
      const int tl = kTiles ? idx / tile_elems : 0, e = idx - tl * tile_elems;
      const float* r0 = s_red + tl * RG * tile_elems + e;
      float v = r0[0];
#pragma unroll
      for (int r = 1; r < RG; ++r) v += r0[r * tile_elems];
      store_out(p, pp, epi, world, epoch, e / T::kNT, (t_first + tl * t_step) * T::kNT + e % T::kNT, v,
                s_epi[e]);
    }
  } else {
    if (RG > 1) {
      for (int idx = threadIdx.x; idx < n_tl * tile_elems; idx += T::kThreads) {
        const int tl = kTiles ? idx / tile_elems : 0, e = idx - tl * tile_elems;
        float* r0 = s_red + tl * RG * tile_elems + e;
        float v = r0[0];
#pragma unroll
        for (int r = 1; r < RG; ++r) v += r0[r * tile_elems];
        r0[0] = v;
      }
    }
    // Split-K over the cluster: every CTA sums a share of its tiles over all
    // ranks' partials in rank order (DSMEM reads), then writes it. The CTAs
    // of a cluster share blockIdx.x, hence the tiles.
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    const unsigned epoch = s_epoch;
    const int rank = (int)cluster.block_rank();
    for (int idx = rank * T::kThreads + threadIdx.x; idx < n_tl * tile_elems;
         idx += T::kThreads * nsplit) {
      const int tl = kTiles ? idx / tile_elems : 0, e = idx - tl * tile_elems;
      const int at = tl * RG * tile_elems + e;
      float v = 0.f;
      for (int r = 0; r < nsplit; ++r) v += cluster.map_shared_rank(s_red, r)[at];
      store_out(p, pp, epi, world, epoch, e / T::kNT, (t_first + tl * t_step) * T::kNT + e % T::kNT, v,
                s_epi[e]);
    }
    cluster.sync();  // keep this CTA's shared memory alive for the readers
  }

  if (world > 0) {
    __syncthreads();
    publish_gathered(p, pp, s_epoch, gridDim.x * gridDim.y);
  }
}


// ---------------------------------------------------------------- instance tables

template <bool B, int MB, int SW, int RG, int OPS>
inline void* gemv_kptr() {
  return reinterpret_cast<void*>(&w4_gemv_kernel<B, MB, SW, RG, OPS>);
}

// The instance for a tile of `sw` strips and `rg` row groups, or nullptr.
template <bool B, int MB, int OPS>
inline void* gemv_pick_tile(int sw, int rg) {
  switch (sw * 16 + rg) {
    case 1 * 16 + 1: return gemv_kptr<B, MB, 1, 1, OPS>();
    case 1 * 16 + 2: return gemv_kptr<B, MB, 1, 2, OPS>();
    case 1 * 16 + 4: return gemv_kptr<B, MB, 1, 4, OPS>();
    case 1 * 16 + 8: return gemv_kptr<B, MB, 1, 8, OPS>();
    case 2 * 16 + 1: return gemv_kptr<B, MB, 2, 1, OPS>();
    case 2 * 16 + 2: return gemv_kptr<B, MB, 2, 2, OPS>();
    case 2 * 16 + 4: return gemv_kptr<B, MB, 2, 4, OPS>();
    case 4 * 16 + 1: return gemv_kptr<B, MB, 4, 1, OPS>();
    case 4 * 16 + 2: return gemv_kptr<B, MB, 4, 2, OPS>();
    default: return nullptr;
  }
}

// The plain instances with several tiles per CTA column also come in tiles
// of 16 compute warps (2 strips x 8 row groups, 4 x 4): one CTA per SM that
// streams its columns through a deep ring.
template <bool B, int MB>
inline void* gemv_pick_stream_tile(int sw, int rg) {
  switch (sw * 16 + rg) {
    case 2 * 16 + 8: return gemv_kptr<B, MB, 2, 8, kOpsPlainTiles>();
    case 4 * 16 + 4: return gemv_kptr<B, MB, 4, 4, kOpsPlainTiles>();
    default: return gemv_pick_tile<B, MB, kOpsPlainTiles>(sw, rg);
  }
}

// Instances by operation set: plain (w4_gemv.cu), generic and plain with
// several tiles per CTA column (w4_gemv_ops.cu), and the fused decode
// combinations, bf16 activations with up to 8 batch rows (w4_gemv_fused.cu).
void* gemv_kernel_plain(int bf16, int mb, int sw, int rg);
void* gemv_kernel_generic(int bf16, int mb, int sw, int rg);
void* gemv_kernel_plain_tiles(int bf16, int mb, int sw, int rg);
void* gemv_kernel_peer(int bf16, int mb, int sw, int rg);
void* gemv_kernel_fused(int ops, int sw, int rg);

}  // namespace w4
