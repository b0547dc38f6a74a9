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
//
// Work split: a launch covers a region of output tiles in row-major order
// (blockIdx.x) and may cut K into up to 16 slices (blockIdx.z), the slices of
// a tile forming a thread-block cluster. A sliced CTA leaves its fp32
// accumulators in shared memory (the freed operand rings) and every rank then
// sums a band of the tile's rows over all ranks in rank order (DSMEM), so the
// result does not depend on scheduling. The host uses slices for grids of
// too few tiles, and for the last few tiles of a grid that would otherwise
// leave most SMs idle in a final wave (a second, programmatically dependent
// launch that runs while the first one's last wave finishes).
#include "w4_internal.h"
#include "w4_ptx.cuh"

#include <cooperative_groups.h>

#include <algorithm>

namespace cg = cooperative_groups;

namespace w4 {

namespace {

constexpr int kUM = 128;          // MMA M (rows of one accumulator)
constexpr int kBMMax = 2 * kUM;   // rows of Y per CTA: up to two accumulators share a W tile
constexpr int kBK = 64;           // k per ring stage (one 128-byte swizzle row of fp16)
constexpr int kBStages = 3;       // dequantised W buffers
constexpr int kDqWarps = 8;       // dequant (and epilogue) warps
constexpr int kMmaWarp = 1 + kDqWarps;
constexpr int kGemmThreads = 32 * (kMmaWarp + 1);  // warp 0 TMA, 1..8 dequant, 9 MMA
constexpr int kErrGemmWait = 7;

struct GemmParams {
  void* y;
  int M, K, N;
  int x_bf16, y_bf16;
  int* err;
  // output tiles of this launch: blockIdx.x = t is tile (m_tile0 + t / ntx,
  // n_tile0 + t % ntx) in units of the instance's rows and columns
  int m_tile0, n_tile0, ntx;
  int ksplit;       // K slices (gridDim.z, one cluster per tile when > 1)
  int wait_at_end;  // a launch overlapping the previous one on the stream
                    // completes only after it (griddepcontrol.wait at exit)
};

// Tile of BN columns (MMA N = BN, 128 or 256) and its shared memory layout
// (base 1024-aligned): X ring, B buffers, packed ring, scale ring, then the
// barriers and the tensor-memory address.
template <int BN, int NACC>
struct GemmShape {
  // TMA ring: 3 slots of 32 KB X tiles with two accumulators; 4 slots of
  // 16 KB with one (the same bytes in flight, one more stage of latency cover)
  static constexpr int kStages = NACC == 1 ? 4 : 3;
  static constexpr int kNumBars = 2 * kStages + 2 * kBStages + 1;
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
  // K slices: the fp32 partial tile (rows padded by 4 floats against bank
  // conflicts) reuses the X and B rings, free once the accumulators are final
  static constexpr int kPitch = BN + 4;
  static constexpr bool kCanSplit = kBM * kPitch * 4 <= kOffPk;
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
  uint64_t* empty_tma = full_tma + S::kStages;        // dequant read the words, MMA read X
  uint64_t* full_b = empty_tma + S::kStages;          // B buffer written
  uint64_t* empty_b = full_b + kBStages;           // MMA read the B buffer
  uint64_t* acc_full = empty_b + kBStages;         // accumulator final
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + S::kOffTmem);
  int* abort_flag = reinterpret_cast<int*>(base + S::kOffTmem + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = (int)blockIdx.x;
  const int n0 = (p.n_tile0 + t % p.ntx) * BN, m0 = (p.m_tile0 + t / p.ntx) * S::kBM;
  // this CTA's K slice: 64-k stages [kt0, kt0 + KT)
  const int KT_all = p.K / kBK;
  const int kt0 = (int)((long long)blockIdx.z * KT_all / p.ksplit);
  const int KT = (int)((long long)(blockIdx.z + 1) * KT_all / p.ksplit) - kt0;
  grid_launch_dependents();  // a dependent launch may fill the SMs this grid frees

  if (threadIdx.x == 0) {
    for (int i = 0; i < S::kStages; ++i) {
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
        const int s = kt % S::kStages;
        if (kt >= S::kStages && !mbar_wait(&empty_tma[s], ((kt / S::kStages) & 1) ^ 1u)) {
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
      for (int j = issued - S::kStages > 0 ? issued - S::kStages : 0; j < issued; ++j)
        if (!mbar_wait(&full_tma[j % S::kStages], (j / S::kStages) & 1)) give_up(kErrDrainWait);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA
    if (lane == 0) {
      constexpr uint32_t idesc = f16_idesc(kBF16 ? 1 : 0, kUM, BN);
      int done = 0;
      for (int kt = 0; kt < KT && !stopped(); ++kt) {
        const int s = kt % S::kStages, sb = kt % kBStages;
        if (!mbar_wait(&full_tma[s], (kt / S::kStages) & 1) ||
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
      const int s = kt % S::kStages, sb = kt % kBStages;
      if (!mbar_wait(&full_tma[s], (kt / S::kStages) & 1) ||
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
    if (p.ksplit > 1) {
      // K slice: this warp's 32 rows of its accumulator -> the fp32 partial tile
      if constexpr (S::kCanSplit) {
        const int q = warp & 3, half = (warp - 1) / 4;
        if (!stopped() && half < NACC) {
          float* prow = reinterpret_cast<float*>(base) + (size_t)(half * kUM + 32 * q + lane) * S::kPitch;
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(tmem_d + ((uint32_t)(32 * q) << 16) + half * BN + 32 * c, r);
#pragma unroll
            for (int v = 0; v < 8; ++v)
              *reinterpret_cast<uint4*>(prow + 32 * c + 4 * v) =
                  make_uint4(r[4 * v], r[4 * v + 1], r[4 * v + 2], r[4 * v + 3]);
          }
        }
      }
    } else if (!stopped()) {
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
  if constexpr (S::kCanSplit) {
    if (p.ksplit > 1) {
      // rank r writes rows [r*R/S, (r+1)*R/S) of the tile, each the sum of
      // every rank's partial in rank order
      cg::cluster_group cluster = cg::this_cluster();
      cluster.sync();
      const int rank = (int)blockIdx.z;
      const int r0 = rank * S::kBM / p.ksplit, r1 = (rank + 1) * S::kBM / p.ksplit;
      constexpr int kC4 = BN / 4;
      const float* part = reinterpret_cast<const float*>(base);
      for (int i = threadIdx.x; i < (r1 - r0) * kC4; i += kGemmThreads) {
        const int row = r0 + i / kC4, c4 = i - (i / kC4) * kC4;
        const int at = row * S::kPitch + 4 * c4;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int rr = 0; rr < p.ksplit; ++rr) {
          const float4 v = *reinterpret_cast<const float4*>(cluster.map_shared_rank(part + at, rr));
          acc.x += v.x;
          acc.y += v.y;
          acc.z += v.z;
          acc.w += v.w;
        }
        const int grow = m0 + row, gcol = n0 + 4 * c4;
        if (grow < p.M && gcol < p.N) {
          uint2 o;
          if (p.y_bf16) {
            const __nv_bfloat162 a = __floats2bfloat162_rn(acc.x, acc.y);
            const __nv_bfloat162 b = __floats2bfloat162_rn(acc.z, acc.w);
            o = make_uint2(*reinterpret_cast<const uint32_t*>(&a),
                           *reinterpret_cast<const uint32_t*>(&b));
          } else {
            const __half2 a = __floats2half2_rn(acc.x, acc.y);
            const __half2 b = __floats2half2_rn(acc.z, acc.w);
            o = make_uint2(*reinterpret_cast<const uint32_t*>(&a),
                           *reinterpret_cast<const uint32_t*>(&b));
          }
          *reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.y) + (size_t)grow * p.N + gcol) = o;
        }
      }
      cluster.sync();  // the other ranks' reads of this CTA's partial are done
    }
  }
  if (warp == kMmaWarp) {
    // every MMA has completed (acc_full) before its tensor memory is freed
    if (lane == 0 && !mbar_wait(acc_full, 0)) give_up(kErrGemmWait);
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d),
                 "r"(S::kTmemCols)
                 : "memory");
  }
  if (p.wait_at_end) grid_dependency_wait();
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
  } ks[8] = {{gemm_fn<false, 128, 1>(), GemmShape<128, 1>::kSmem},
             {gemm_fn<true, 128, 1>(), GemmShape<128, 1>::kSmem},
             {gemm_fn<false, 256, 1>(), GemmShape<256, 1>::kSmem},
             {gemm_fn<true, 256, 1>(), GemmShape<256, 1>::kSmem},
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

namespace {

// One launch of a prepared plan: the instance, its tile region and K slices.
struct GemmLaunch {
  int bn, nacc;
  int m_tile0, n_tile0, ntx, tiles;
  int ksplit;
  bool after_previous;  // programmatic dependent launch, waits for it at exit
};

void* gemm_instance(int bf16, int bn, int nacc, size_t* smem) {
  if (bn == 256 && nacc == 2) {
    *smem = GemmShape<256, 2>::kSmem;
    return bf16 ? gemm_fn<true, 256, 2>() : gemm_fn<false, 256, 2>();
  }
  if (bn == 256) {
    *smem = GemmShape<256, 1>::kSmem;
    return bf16 ? gemm_fn<true, 256, 1>() : gemm_fn<false, 256, 1>();
  }
  if (nacc == 2) {
    *smem = GemmShape<128, 2>::kSmem;
    return bf16 ? gemm_fn<true, 128, 2>() : gemm_fn<false, 128, 2>();
  }
  *smem = GemmShape<128, 1>::kSmem;
  return bf16 ? gemm_fn<true, 128, 1>() : gemm_fn<false, 128, 1>();
}

// The launches of one GEMM (at most two). split_k > 0 forces one launch of
// 128 x 256 tiles (one accumulator) cut into that many K slices.
int gemm_plan(int M, int K, int N, int sms, int split_k, GemmLaunch* out) {
  const int kt = K / kBK;
  const int nt128 = (N + 127) / 128;
  // the K-sliced tile: 128 rows x 256 columns (its partial tile fits the
  // freed rings; two accumulators of 256 columns would not)
  const int nt256 = (N + 255) / 256, mt1 = (M + kUM - 1) / kUM;
  if (split_k > 0) {
    out[0] = GemmLaunch{256, 1, 0, 0, nt256, nt256 * mt1, std::min(split_k, kt), false};
    return 1;
  }
  int nacc = 2;
  const int bn = gemm_tile(M, N, sms, &nacc);
  const int bm = nacc * kUM;
  const int ntx = (N + bn - 1) / bn, mtx = (M + bm - 1) / bm;
  const int tiles = ntx * mtx;
  // A grid of fewer tiles than SMs is not cut along K: measured on 2048 x
  // 8960 x 1536 (96 tiles), three K slices over 288 CTAs took 118-128 us
  // against 96 us for the 96 whole tiles (each slice's stages ran at half the
  // rate).
  if (tiles >= sms && bn == 256 && nacc == 2) {
    // a last wave of a few tiles: those tiles go to a second launch as
    // 128-column tiles cut into K slices, spread over the SMs the first
    // launch frees
    const int rem = tiles % sms;
    if (rem > 0 && rem * 4 <= sms && rem <= ntx) {
      const int n_lo = (ntx - rem) * 2;  // first 128-column tile of the remainder
      const int nrx = nt128 - n_lo;
      const int s = std::max(1, std::min(8, std::min(sms / nrx, kt / 4)));
      out[0] = GemmLaunch{256, 2, 0, 0, ntx, tiles - rem, 1, false};
      out[1] = GemmLaunch{128, 2, mtx - 1, n_lo, nrx, nrx, s, true};
      return 2;
    }
  }
  out[0] = GemmLaunch{bn, nacc, 0, 0, ntx, tiles, 1, false};
  return 1;
}

}  // namespace

int launch_gemm(const void* x, int x_bf16, const int32_t* packed, const void* scales, void* y,
                int y_bf16, int M, int K, int N, int split_k, cudaStream_t stream) {
  int dev = 0;
  int st = current_device(&dev);
  if (st != W4_OK) return st;
  const DeviceInfo& di = device_info(dev);
  GemmLaunch plan[2];
  const int n = gemm_plan(M, K, N, di.sm_count > 0 ? di.sm_count : 148, split_k, plan);
  for (int i = 0; i < n; ++i) {
    const GemmLaunch& L = plan[i];
    const int BM = L.nacc * kUM;
    CUtensorMap tm_x, tm_w, tm_s;
    if (!encode_2d(&tm_x,
                   x_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                   x, (uint64_t)K, (uint64_t)M, kBK, (uint32_t)BM, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_2d(&tm_w, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, packed, (uint64_t)N,
                   (uint64_t)(K / 8), (uint32_t)L.bn, kBK / 8, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode_2d(&tm_s, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, scales, (uint64_t)N,
                   (uint64_t)(K / 128), (uint32_t)L.bn, 1, CU_TENSOR_MAP_SWIZZLE_NONE))
      return fail(W4_ERR_CUDA, "cuTensorMapEncodeTiled failed for w4_gemm M=%d K=%d N=%d", M, K,
                  N);
    GemmParams p;
    p.y = y;
    p.M = M;
    p.K = K;
    p.N = N;
    p.x_bf16 = x_bf16;
    p.y_bf16 = y_bf16;
    p.err = di.err_word;
    p.m_tile0 = L.m_tile0;
    p.n_tile0 = L.n_tile0;
    p.ntx = L.ntx;
    p.ksplit = L.ksplit;
    p.wait_at_end = L.after_previous ? 1 : 0;
    size_t smem = 0;
    void* fn = gemm_instance(x_bf16, L.bn, L.nacc, &smem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)L.tiles, 1, (unsigned)L.ksplit);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attrs[2];
    unsigned na = 0;
    if (L.ksplit > 1) {
      attrs[na].id = cudaLaunchAttributeClusterDimension;
      attrs[na].val.clusterDim.x = 1;
      attrs[na].val.clusterDim.y = 1;
      attrs[na].val.clusterDim.z = (unsigned)L.ksplit;
      ++na;
    }
    if (L.after_previous) {
      attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attrs[na].val.programmaticStreamSerializationAllowed = 1;
      ++na;
    }
    cfg.attrs = attrs;
    cfg.numAttrs = na;
    void* args[] = {&tm_x, &tm_w, &tm_s, &p};
    cudaError_t e = cudaLaunchKernelExC(&cfg, fn, args);
    if (e != cudaSuccess) return cuda_fail(e, "w4_gemm launch");
  }
  return W4_OK;
}

}  // namespace w4
