// w4_ptx.cuh - thin inline-PTX helpers for sm_100a used by the W4A16 kernels:
// mbarriers with bounded waits, TMA tile loads, legacy-pipe mma.sync,
// LOP3-based nibble unpack and programmatic-dependent-launch controls.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace w4 {

// A wait on an mbarrier gives up after this long and reports an error instead
// of spinning forever (the kernels then drain their copies and return).
constexpr unsigned long long kWaitLimitNs = 1000ull * 1000ull * 1000ull;  // 1 s
// Upper bound on one parked try_wait (the bounded wait re-checks its clock
// between tries, so the 1 s limit still holds).
constexpr uint32_t kSuspendHintNs = 20000;  // 20 us

// Device-side error word; kernels set it when a bounded wait gives up.
enum : int { kErrNone = 0, kErrFullWait = 1, kErrEmptyWait = 2, kErrDrainWait = 3 };

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// One potentially blocking test of the phase. The suspend-time hint lets the
// hardware park the thread until the phase completes (or the hint's time
// passes) instead of returning at once, so waiting warps do not spin on the
// issue slots the computing warps need.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete. Returns false if it
// did not complete within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
}

// ---------------------------------------------------------------- TMA
// 2-D tiled bulk tensor load into this CTA's shared memory, completion
// signalled on `bar` as transaction bytes. c0 is the innermost coordinate.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- PDL
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- shared loads
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

// ---------------------------------------------------------------- math
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;  // (a & b) | c
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint32_t fma_f16x2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint32_t fma_bf16x2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Unpacks the 8 nibbles of one packed word into four 16-bit pairs of
// small exact integers, with one LOP3 per pair: the nibble is OR-ed into the
// mantissa of a constant whose mantissa unit is one, turning it into a float
// without a conversion instruction.
//   fp16: h[0] = (1024+q0, 1024+q4)        h[1] = (1024+16q1, 1024+16q5)
//         h[2] = (1024+q2, 1024+q6)        h[3] = (1024+16q3, 1024+16q7)
//   bf16: h[i] = (128+q_i, 128+q_{i+4})    (the 16q form does not fit bf16)
// (first element in the low half). The constant and the zero point are not
// removed here: the GEMV folds them into one per-(group, row) correction, and
// the fp16 "16q" slots meet activations pre-scaled by 1/16.
template <bool kBF16>
__device__ __forceinline__ void unpack_nibbles(uint32_t w, uint32_t (&h)[4]) {
  if constexpr (!kBF16) {
    constexpr uint32_t kMagic = 0x64006400u;  // 1024 | 1024
    const uint32_t w8 = w >> 8;
    h[0] = lop3_and_or(w, 0x000F000Fu, kMagic);
    h[1] = lop3_and_or(w, 0x00F000F0u, kMagic);
    h[2] = lop3_and_or(w8, 0x000F000Fu, kMagic);
    h[3] = lop3_and_or(w8, 0x00F000F0u, kMagic);
  } else {
    constexpr uint32_t kMagic = 0x43004300u;  // 128 | 128
    h[0] = lop3_and_or(w, 0x000F000Fu, kMagic);
    h[1] = lop3_and_or(w >> 4, 0x000F000Fu, kMagic);
    h[2] = lop3_and_or(w >> 8, 0x000F000Fu, kMagic);
    h[3] = lop3_and_or(w >> 12, 0x000F000Fu, kMagic);
  }
}

// Per-element offsets the unpacked values carry, for the correction term:
//   fp16 low-nibble slots (h[0], h[2]) hold (q - 8) + 1032 against x,
//   fp16 high-nibble slots (h[1], h[3]) hold 16 * ((q - 8) + 72) against x/16,
//   bf16 slots hold (q - 8) + 136 against x.
constexpr float kF16LowOffset = 1032.0f;
constexpr float kF16HighOffset = 72.0f * 16.0f;  // applied to the staged x/16
constexpr float kBF16Offset = 136.0f;

// D += A(16x16, row) * B(16x8, col), fp32 accumulate.
template <bool kBF16>
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  if constexpr (!kBF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

}  // namespace w4
