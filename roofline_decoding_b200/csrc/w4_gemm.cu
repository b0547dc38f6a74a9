// w4_gemm.cu - W4A16 GEMM on the 5th-generation tensor cores (tcgen05) for
// the prefill rows of W4Linear.
//
// Y[M, N] = X[M, K] @ W[K, N], W = dequantize_v1(packed, scales): the
// operation the reference runs for more than 8 rows as dequantize_v1 (an
// fp16 [K, N] copy of the weights, roofline/kernels.py:77-90) followed by an
// fp32 matmul (scripts/decode_loop.py:51-55). Here the dequantised tile never
// leaves shared memory:
//   TMA warp     : X tiles [up to 256 rows x 64 k] (128B swizzle, the
//                  canonical K-major layout the MMA reads) and the packed
//                  words and scales of the W tile (128 or 256 columns),
//                  through a 3-slot ring;
//   8 dequant warps: expand each packed word into 8 fp16 (q - 8) * s values
//                  - bit-identical to dequantize_v1 - and write them K-major,
//                  128B-swizzled, into one of three B buffers;
//   MMA warp     : one thread issues tcgen05.mma (M = 128, N = 128 or 256,
//                  K = 16, fp32 accumulate in tensor memory), four per 64-k
//                  stage for each of the tile's one or two 128-row halves
//                  (both halves share one dequantised B tile), and commits to
//                  the ring's mbarriers;
//   epilogue     : the dequant warps read the accumulators with tcgen05.ld
//                  and store Y (fp16 or bf16).
// bf16 activations use bf16 weights bf16((q - 8) * s) (one rounding of the
// fp32 product; the reference has no bf16 path). Every wait is bounded; a
// CTA that gives up sets the device error word, drains its copies and
// frees its tensor memory.
#include "w4_internal.h"
#include "w4_ptx.cuh"

#include <algorithm>

namespace w4 {

namespace {

constexpr int kUM = 128;          // MMA M (rows of one accumulator)
constexpr int kBMMax = 2 * kUM;   // rows of Y per CTA: up to two accumulators share a W tile
constexpr int kBK = 64;           // k per ring stage (one 128-byte swizzle row of fp16)
constexpr int kStages = 3;        // TMA ring
constexpr int kBStages = 3;       // dequantised W buffers
constexpr int kDqWarps = 8;       // dequant (and epilogue) warps
constexpr int kMmaWarp = 1 + kDqWarps;
constexpr int kGemmThreads = 32 * (kMmaWarp + 1);  // warp 0 TMA, 1..8 dequant, 9 MMA
constexpr int kNumBars = 2 * kStages + 2 * kBStages + 1;
constexpr int kErrGemmWait = 7;

struct GemmParams {
  void* y;
  int M, K, N;
  int x_bf16, y_bf16;
  int* err;
};

// Tile of BN columns (MMA N = BN, 128 or 256) and its shared memory layout
// (base 1024-aligned): X ring, B buffers, packed ring, scale ring, then the
// barriers and the tensor-memory address.
template <int BN, int NACC>
struct GemmShape {
  static constexpr int kBM = NACC * kUM;                 // rows of Y per CTA
  static constexpr int kXBytes = kBM * kBK * 2;          // 16 or 32 KB
  static constexpr int kBBytes = BN * kBK * 2;           // 16 or 32 KB
  static constexpr int kPkBytes = (kBK / 8) * BN * 4;    // packed words of a stage
  static constexpr int kScBytes = BN * 2;                // scales of a stage
  static constexpr int kTmemCols = NACC * BN;            // fp32 accumulators
  static constexpr int kOffX = 0;
  static constexpr int kOffB = kOffX + kStages * kXBytes;
  static constexpr int kOffPk = kOffB + kBStages * kBBytes;
  static constexpr int kOffSc = kOffPk + kStages * kPkBytes;
  static constexpr int kOffBar = kOffSc + kStages * kScBytes;
  static constexpr int kOffTmem = kOffBar + kNumBars * 8;
  static constexpr int kSmem = 1024 + kOffTmem + 16;
  static constexpr int kThreadsPerCol = kDqWarps * 32 / BN;  // dequant threads per column
  static constexpr int kWordsPerThread = (kBK / 8) / kThreadsPerCol;
  static_assert(kOffB % 1024 == 0 && kXBytes % 1024 == 0 && kBBytes % 1024 == 0,
                "swizzled operand tiles start on 1024-byte boundaries");
  static_assert(kOffPk % 128 == 0 && kOffSc % 128 == 0 && kPkBytes % 128 == 0 &&
                    kScBytes % 128 == 0,
                "tensor-copy destinations are 128-byte aligned");
  static_assert(kTmemCols <= 512 && kWordsPerThread * kThreadsPerCol == kBK / 8, "tile");
};

// ---------------------------------------------------------------- tcgen05

// Shared-memory matrix descriptor of a K-major operand tile in the canonical
// 128B-swizzle layout: rows of 128 bytes (64 fp16 of k), 8-row atoms of
// 1024 bytes stacked along M/N. Fields (16-byte units): start address,
// leading byte offset 1 (unused by swizzled K-major), stride byte offset 64
// (1024 bytes between atoms), version 1, layout type 2 (128B swizzle).
__device__ __forceinline__ uint64_t kmajor_sw128_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)64u << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// Instruction descriptor of kind::f16: fp32 accumulate, A and B of one type
// (0 fp16, 1 bf16), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t f16_idesc(int bf16, int m, int n) {
  return (1u << 4) | ((uint32_t)bf16 << 7) | ((uint32_t)bf16 << 10) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      :
      : "r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u),
        "r"(0u)
      : "memory");
}

// Arrives once on the mbarrier when every tcgen05 operation this thread
// issued before has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Generic-proxy shared-memory stores become visible to the tensor core's
// (async proxy) reads.
__device__ __forceinline__ void fence_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- dequant

// One packed word (8 consecutive k of one column, nibble i = k 8j + i) to 8
// dequantised 16-bit values in k order: pair (q_2i, q_2i+1) is built by one
// byte permute of the word and its 4-bit shift plus one LOP3 into the
// mantissa of 1024 (fp16) or 128 (bf16); then (q - 8) is exact and the
// scale product is rounded once.
template <bool kBF16>
__device__ __forceinline__ uint4 dequant_word(uint32_t w, uint32_t s2, float sf) {
  const uint32_t y = w >> 4;
  uint32_t h[4];
  h[0] = __byte_perm(w, y, 0x4400);
  h[1] = __byte_perm(w, y, 0x5511);
  h[2] = __byte_perm(w, y, 0x6622);
  h[3] = __byte_perm(w, y, 0x7733);
  uint4 out;
  uint32_t* o = reinterpret_cast<uint32_t*>(&out);
  if constexpr (!kBF16) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t v = lop3_and_or(h[i], 0x000F000Fu, 0x64006400u);  // 1024 + q
      __half2 d = __hsub2(*reinterpret_cast<const __half2*>(&v),
                          __half2half2(__ushort_as_half(0x6408)));   // q - 8 (1032)
      d = __hmul2(d, *reinterpret_cast<const __half2*>(&s2));       // one rounding
      o[i] = *reinterpret_cast<const uint32_t*>(&d);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t v = lop3_and_or(h[i], 0x000F000Fu, 0x43004300u);  // 128 + q
      const float lo = __uint_as_float(v << 16) - 136.0f;                // q - 8, exact
      const float hi = __uint_as_float(v & 0xFFFF0000u) - 136.0f;
      const __nv_bfloat162 d = __floats2bfloat162_rn(lo * sf, hi * sf);  // one rounding
      o[i] = *reinterpret_cast<const uint32_t*>(&d);
    }
  }
  return out;
}

template <bool kBF16, int BN, int NACC>
__global__ void __launch_bounds__(kGemmThreads, 1)
    w4_gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                   const __grid_constant__ CUtensorMap tm_s, const GemmParams p) {
  using S = GemmShape<BN, NACC>;
  extern __shared__ uint8_t smem_gemm[];
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_gemm) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + S::kOffBar);
  uint64_t* full_tma = bars;                       // X + packed + scales landed
  uint64_t* empty_tma = full_tma + kStages;        // dequant read the words, MMA read X
  uint64_t* full_b = empty_tma + kStages;          // B buffer written
  uint64_t* empty_b = full_b + kBStages;           // MMA read the B buffer
  uint64_t* acc_full = empty_b + kBStages;         // accumulator final
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + S::kOffTmem);
  int* abort_flag = reinterpret_cast<int*>(base + S::kOffTmem + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * S::kBM;
  const int KT = p.K / kBK;
  constexpr int kt0 = 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full_tma[i], 1);
      mbar_init(&empty_tma[i], kDqWarps + 1);  // the dequant warps + the MMA commit
    }
    for (int i = 0; i < kBStages; ++i) {
      mbar_init(&full_b[i], kDqWarps);
      mbar_init(&empty_b[i], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {  // tensor memory for the two 128 x 128 fp32 accumulators
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(S::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = *tmem_slot;
  auto give_up = [&](int code) {
    if (p.err) atomicCAS(p.err, 0, code);
    *reinterpret_cast<volatile int*>(abort_flag) = 1;
  };
  auto stopped = [&]() { return *reinterpret_cast<volatile int*>(abort_flag) != 0; };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA
    if (lane == 0) {
      tma_prefetch_desc(&tm_x);
      tma_prefetch_desc(&tm_w);
      tma_prefetch_desc(&tm_s);
      int issued = 0;
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % kStages;
        if (kt >= kStages && !mbar_wait(&empty_tma[s], ((kt / kStages) & 1) ^ 1u)) {
          give_up(kErrGemmWait);
          break;
        }
        if (stopped()) break;
        mbar_arrive_expect_tx(&full_tma[s], S::kXBytes + S::kPkBytes + S::kScBytes);
        const int kg = kt0 + kt;  // stage of the whole K
        tma_load_2d(base + S::kOffX + s * S::kXBytes, &tm_x, &full_tma[s], kg * kBK, m0);
        tma_load_2d(base + S::kOffPk + s * S::kPkBytes, &tm_w, &full_tma[s], n0, kg * (kBK / 8));
        tma_load_2d(base + S::kOffSc + s * S::kScBytes, &tm_s, &full_tma[s], n0, (kg * kBK) / 128);
        ++issued;
      }
      for (int j = issued - kStages > 0 ? issued - kStages : 0; j < issued; ++j)
        if (!mbar_wait(&full_tma[j % kStages], (j / kStages) & 1)) give_up(kErrDrainWait);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA
    if (lane == 0) {
      constexpr uint32_t idesc = f16_idesc(kBF16 ? 1 : 0, kUM, BN);
      int done = 0;
      for (int kt = 0; kt < KT && !stopped(); ++kt) {
        const int s = kt % kStages, sb = kt % kBStages;
        if (!mbar_wait(&full_tma[s], (kt / kStages) & 1) ||
            !mbar_wait(&full_b[sb], (kt / kBStages) & 1)) {
          give_up(kErrGemmWait);
          break;
        }
        tc_fence_after();
        const uint32_t xa = smem_u32(base + S::kOffX + s * S::kXBytes);
        const uint32_t ba = smem_u32(base + S::kOffB + sb * S::kBBytes);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {  // 16 k = 32 bytes along the swizzled row
          const uint64_t bd = kmajor_sw128_desc(ba + kk * 32);
          const uint32_t acc = (kt > 0 || kk > 0) ? 1u : 0u;
          // accumulator a: rows 128a.. (16 KB further per 128 rows), columns a*BN..
#pragma unroll
          for (int a = 0; a < NACC; ++a)
            umma_f16(tmem_d + a * BN, kmajor_sw128_desc(xa + a * kUM * 128 + kk * 32), bd, idesc,
                     acc);
        }
        umma_commit(&empty_tma[s]);
        umma_commit(&empty_b[sb]);
        ++done;
      }
      umma_commit(acc_full);  // after every issued MMA (also when none was issued)
      (void)done;
    }
  } else {
    // ------------------------------------------------------------ dequant
    const int dt = threadIdx.x - 32;
    const int n = dt % BN;                                  // column of the tile
    const int jh = (dt / BN) * S::kWordsPerThread;          // this thread's words of the column
    for (int kt = 0; kt < KT && !stopped(); ++kt) {
      const int s = kt % kStages, sb = kt % kBStages;
      if (!mbar_wait(&full_tma[s], (kt / kStages) & 1) ||
          (kt >= kBStages && !mbar_wait(&empty_b[sb], ((kt / kBStages) & 1) ^ 1u))) {
        give_up(kErrGemmWait);
        break;
      }
      const uint32_t* pk = reinterpret_cast<const uint32_t*>(base + S::kOffPk + s * S::kPkBytes);
      const uint16_t sbits = reinterpret_cast<const uint16_t*>(base + S::kOffSc + s * S::kScBytes)[n];
      const uint32_t s2 = (uint32_t)sbits | ((uint32_t)sbits << 16);
      const float sf = __half2float(__ushort_as_half(sbits));
      uint8_t* brow = base + S::kOffB + sb * S::kBBytes + n * 128;  // row n: 64 k of column n
      uint32_t wv[S::kWordsPerThread];
#pragma unroll
      for (int j = 0; j < S::kWordsPerThread; ++j) wv[j] = pk[(jh + j) * BN + n];
#pragma unroll
      for (int j = 0; j < S::kWordsPerThread; ++j)  // chunk j lands at chunk j ^ (row % 8)
        *reinterpret_cast<uint4*>(brow + (((jh + j) ^ (n & 7)) << 4)) =
            dequant_word<kBF16>(wv[j], s2, sf);
      fence_async_shared();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&full_b[sb]);
        mbar_arrive(&empty_tma[s]);
      }
    }
    // ------------------------------------------------------------ epilogue
    if (!mbar_wait(acc_full, 0)) give_up(kErrGemmWait);
    tc_fence_after();
    if (!stopped()) {
      const int q = warp & 3;            // this warp's 32-lane slice of tensor memory
      const int half = (warp - 1) / 4;   // which accumulator (rows 0..127 or 128..255)
      if (half >= NACC) goto epilogue_done;
      const int row = m0 + half * kUM + 32 * q + lane;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem_d + ((uint32_t)(32 * q) << 16) + half * BN + 32 * c, r);
        if (row < p.M && n0 + 32 * c < p.N) {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.y) +
                                                (size_t)row * p.N + n0 + 32 * c);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 o;
            uint32_t* oi = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float a = __uint_as_float(r[8 * v + 2 * e]);
              const float b = __uint_as_float(r[8 * v + 2 * e + 1]);
              if (p.y_bf16) {
                const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
                oi[e] = *reinterpret_cast<const uint32_t*>(&h);
              } else {
                const __half2 h = __floats2half2_rn(a, b);
                oi[e] = *reinterpret_cast<const uint32_t*>(&h);
              }
            }
            dst[v] = o;
          }
        }
      }
    }
  epilogue_done:
    tc_fence_before();
  }
  __syncthreads();
  if (warp == kMmaWarp) {
    // every MMA has completed (acc_full) before its tensor memory is freed
    if (lane == 0 && !mbar_wait(acc_full, 0)) give_up(kErrGemmWait);
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d),
                 "r"(S::kTmemCols)
                 : "memory");
  }
}

bool encode_2d(CUtensorMap* map, CUtensorMapDataType dt, int elem, const void* gaddr,
               uint64_t inner, uint64_t outer, uint32_t box_inner, uint32_t box_outer,
               CUtensorMapSwizzle swz) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * (uint64_t)elem};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, dt, 2, const_cast<void*>(gaddr), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

template <bool B, int BN, int NACC>
void* gemm_fn() {
  return reinterpret_cast<void*>(&w4_gemm_kernel<B, BN, NACC>);
}

int gemm_init_device(const DeviceInfo& di) {
  struct K {
    void* fn;
    int smem;
  } ks[6] = {{gemm_fn<false, 128, 1>(), GemmShape<128, 1>::kSmem},
             {gemm_fn<true, 128, 1>(), GemmShape<128, 1>::kSmem},
             {gemm_fn<false, 128, 2>(), GemmShape<128, 2>::kSmem},
             {gemm_fn<true, 128, 2>(), GemmShape<128, 2>::kSmem},
             {gemm_fn<false, 256, 2>(), GemmShape<256, 2>::kSmem},
             {gemm_fn<true, 256, 2>(), GemmShape<256, 2>::kSmem}};
  for (const K& k : ks) {
    if ((size_t)k.smem > (size_t)di.max_smem_optin)
      return fail(W4_ERR_UNSUPPORTED, "w4_gemm needs %d B of shared memory", k.smem);
    cudaError_t e = cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, k.smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(w4_gemm smem)");
    e = cudaFuncSetAttribute(k.fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(w4_gemm carveout)");
  }
  return W4_OK;
}

// Tile width: 256 columns halve the re-reads of X per FLOP; 128 when a
// 256-wide grid would not cover the SMs.
// Two accumulators (256 rows) share every dequantised W tile, which halves
// the dequantisation per FLOP; one only when M fits 128 rows.
static int gemm_tile(int M, int N, int sms, int* nacc) {
  const long long m2 = (M + kBMMax - 1) / kBMMax;
  *nacc = M <= kUM ? 1 : 2;
  if (*nacc == 2 && (N % 256 == 0 || N > 1024) && (long long)((N + 255) / 256) * m2 >= sms)
    return 256;
  return 128;
}

int launch_gemm(const void* x, int x_bf16, const int32_t* packed, const void* scales, void* y,
                int y_bf16, int M, int K, int N, cudaStream_t stream) {
  int dev = 0;
  int st = current_device(&dev);
  if (st != W4_OK) return st;
  const DeviceInfo& di = device_info(dev);
  int nacc = 2;
  const int BN = gemm_tile(M, N, di.sm_count > 0 ? di.sm_count : 148, &nacc);
  const int BM = nacc * kUM;
  CUtensorMap tm_x, tm_w, tm_s;
  if (!encode_2d(&tm_x, x_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                 2, x, (uint64_t)K, (uint64_t)M, kBK, (uint32_t)BM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_2d(&tm_w, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, packed, (uint64_t)N, (uint64_t)(K / 8),
                 (uint32_t)BN, kBK / 8, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !encode_2d(&tm_s, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, scales, (uint64_t)N,
                 (uint64_t)(K / 128), (uint32_t)BN, 1, CU_TENSOR_MAP_SWIZZLE_NONE))
    return fail(W4_ERR_CUDA, "cuTensorMapEncodeTiled failed for w4_gemm M=%d K=%d N=%d", M, K, N);
  GemmParams p;
  p.y = y;
  p.M = M;
  p.K = K;
  p.N = N;
  p.x_bf16 = x_bf16;
  p.y_bf16 = y_bf16;
  p.err = di.err_word;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((N + BN - 1) / BN), (unsigned)((M + BM - 1) / BM), 1);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.stream = stream;
  void* fn;
  if (BN == 256) {
    cfg.dynamicSmemBytes = GemmShape<256, 2>::kSmem;
    fn = x_bf16 ? gemm_fn<true, 256, 2>() : gemm_fn<false, 256, 2>();
  } else if (nacc == 2) {
    cfg.dynamicSmemBytes = GemmShape<128, 2>::kSmem;
    fn = x_bf16 ? gemm_fn<true, 128, 2>() : gemm_fn<false, 128, 2>();
  } else {
    cfg.dynamicSmemBytes = GemmShape<128, 1>::kSmem;
    fn = x_bf16 ? gemm_fn<true, 128, 1>() : gemm_fn<false, 128, 1>();
  }
  void* args[] = {&tm_x, &tm_w, &tm_s, &p};
  cudaError_t e = cudaLaunchKernelExC(&cfg, fn, args);
  return e == cudaSuccess ? W4_OK : cuda_fail(e, "w4_gemm launch");
}

}  // namespace w4
