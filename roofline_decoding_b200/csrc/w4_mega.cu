// w4_mega.cu - a whole batch-1 greedy decode step as one persistent kernel.
//
// The step of scripts/decode_loop.py:106-124 (embedding, per layer RMSNorm ->
// q|k|v -> RoPE + attention -> o -> RMSNorm -> gate|up -> SwiGLU -> down,
// final RMSNorm, tied lm_head, argmax) run by one cooperative grid of one CTA
// per SM instead of 142 dependent launches.
//
// Why one kernel: at batch 1 every linear is a few MB, and a dependent launch
// costs ~2-6 us of critical path before its first byte arrives, so the
// launch chain, not HBM, set the step time. Here each CTA's producer warp
// streams the packed weights of every layer through one TMA ring without
// stopping at phase boundaries (the weights do not depend on the
// activations), and the consumer warps wait only on grid barriers for the
// activations. The phases of a layer:
//   QKV   x = rmsnorm(h) (h = embedding row, or h1 + down partials), GEMV
//         items write fp32 partials
//   ATTN  q/k/v = bf16(partials + bias), RoPE, KV write, split-KV attention
//         over positions 0..pos, per split (m, l, o) partials
//   O     x = merged attention, GEMV items write fp32 partials
//   GU    x = rmsnorm(h1), h1 = h0 + o partials
//   DOWN  x = silu(gate) * up from the gate|up partials
// and a final LM phase (rmsnorm(h), lm_head rows through the same ring,
// argmax by a 64-bit atomicMax, last CTA advances token and position).
// Whatever a phase needs that does not depend on the previous phase (norm
// weights, the q|k|v bias, RoPE factors, the cached K/V rows) is loaded before
// the grid barrier, so only the activation round trip is on the critical path.
//
// GEMV items: a 32-column strip of the output and a range of K groups (128
// rows); with split > 1 the partials of one strip are summed in a fixed order
// by the consumer of the next phase, so the step is deterministic. The inner
// product is the swap-AB mma.sync of w4_gemv.cu (LOP3 unpack, beta-folded
// zero point, scale per group in fp32).
#include "w4_internal.h"
#include "w4_ptx.cuh"

#include <algorithm>

namespace w4 {

namespace {

constexpr int kMegaConsumerWarps = 8;
constexpr int kNC = kMegaConsumerWarps * 32;             // consumer threads
constexpr int kMegaThreads = kNC + 32;                   // + producer warp
constexpr int kGroupsPerStage = 12;                      // K groups per ring stage
constexpr int kGroupBytes = 16 * 128;                    // 16 packed rows x 32 int32
constexpr int kScaleGroupBytes = 32 * 2;                 // 32 fp16 scales
constexpr int kSlotBytes = kGroupsPerStage * kGroupBytes;  // 24 KB
constexpr int kSlotScaleBytes = kGroupsPerStage * kScaleGroupBytes;  // multiple of 128
constexpr int kSlots = 7;
constexpr int kMaxStagedGroups = 32;   // x staged per CTA and phase: 4096 activations
constexpr int kMaxItems = 4;           // GEMV items per CTA and phase
constexpr int kMaxPartSplit = 3;       // K splits of a GEMV: partial loads are issued together
constexpr int kAttnTileM = 32;         // positions per attention tile
constexpr int kHD = 128;               // head_dim (= K group)
constexpr int kKPitchM = kHD + 8;      // bf16 per K row: 16-byte rows, 4-bank skew
constexpr int kQPitchM = kHD + 4;      // floats per q row
constexpr int kMaxGroupHeads = 8;      // q heads per KV head
constexpr int kMaxAttnSplits = 16;
constexpr int kWorkBytes = 44 * 1024;  // per-phase scratch (aliased by phase type)
constexpr int kBarCounters = 8;        // grid-barrier arrival counters, 128 B apart

constexpr int kErrBarrier = 4;  // a grid barrier wait gave up
constexpr int kErrAlign = 5;    // a copy destination broke its alignment rule (not issued)

__device__ __forceinline__ float bfm(uint16_t v) { return __uint_as_float((uint32_t)v << 16); }
__device__ __forceinline__ uint16_t to_bfm(float v) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}
__device__ __forceinline__ float rbfm(float v) { return bfm(to_bfm(v)); }

__device__ __forceinline__ uint32_t order_key_m(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ void bulk_load_m(void* dst, const void* src, uint32_t bytes,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 16-byte asynchronous global -> shared copy (L2 only) and its completion.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Named barrier of the consumer warps. It is the aligned form: every call
// site must be reached by whole warps.
__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"r"(kNC) : "memory");
}

// bf16 SwiGLU of the staged activation: round(round(silu(g)) * u)
__device__ __forceinline__ float swiglu(float g, float u) {
  return rbfm(rbfm(g / (1.0f + __expf(-g))) * u);
}

}  // namespace

// One GEMV of the step, stacked over layers: packed [layers * K/8, N],
// scales [layers * K/128, N].
struct MegaGemv {
  int N, K, groups, split, gps, strips, items;
  int bg;  // K groups per ring stage: one box of 16*bg packed rows and one of bg scale rows
};

// Tensor maps of the four stacked GEMVs: packed words (box 32 x 16 rows,
// 128B swizzle) and scales (box 32 x 1 group).
struct alignas(64) MegaMaps {
  CUtensorMap w[4];
  CUtensorMap s[4];
};

struct MegaParams {
  int layers, hidden, inter, heads, kv_heads, vocab, max_seq;
  int group;        // q heads per KV head
  int attn_splits;  // position splits per KV head
  int lm_rows;      // lm_head rows per ring stage
  float eps, scale;
  MegaGemv g[4];    // 0 qkv, 1 o, 2 gate|up, 3 down
  const uint16_t* qkv_bias;   // [layers, n_qkv]
  const uint16_t* in_norm;    // [layers, hidden]
  const uint16_t* post_norm;  // [layers, hidden]
  const uint16_t* final_norm;
  const uint16_t* embed;      // [vocab, hidden], also the lm_head
  const uint16_t* cos_t;      // [max_seq, 128]
  const uint16_t* sin_t;
  uint16_t* k_cache;          // [layers, kv_heads, max_seq, 128]
  uint16_t* v_cache;
  const int64_t* prompt;
  const int64_t* prompt_len;
  int64_t* token;
  int64_t* pos;
  uint16_t* logits;           // [vocab] or null
  // scratch (zeroed once by the caller; the step leaves its counters zeroed)
  unsigned* bar;              // kBarCounters arrival counters, 32 words apart
  unsigned* done;             // CTAs finished with the lm_head
  unsigned long long* best;   // argmax key
  uint16_t* h0;               // [hidden] layer input (written by CTA 0)
  uint16_t* h1;               // [hidden] after the attention residual
  float* part[4];             // [split, N] GEMV partials per phase kind
  float* pattn;               // [kv_heads, attn_splits, group * (2 + 128)]
  int* err;
};

namespace {

enum StageSrc : int { kSrcEmbed = 0, kSrcH1Down = 1, kSrcH0O = 2 };

// Shared memory: [ring kSlots x 24 KB][ring scales][work area][barriers]
struct MegaSmem {
  uint8_t* w;       // weights / lm rows
  uint8_t* sc;      // scales
  uint8_t* work;    // phase scratch
  uint64_t* full;
  uint64_t* empty;
  int* abort_flag;
};

// Work-area layout for GEMV phases.
//   xsrc  bf16 [2048]               transformed activations (absolute k index)
//   xs    bf16 [32 groups * 128]    staged x in MMA k order
//   beta  f32  [32]
//   red   f32  [4 items][8 warps][32]
//   misc  f32  [16]
constexpr int kXsrcOff = 0;
constexpr int kXsOff = kXsrcOff + 2048 * 2;
constexpr int kBetaOff = kXsOff + kMaxStagedGroups * 256 + 16;
constexpr int kRedOff = (kBetaOff + kMaxStagedGroups * 4 + 15) / 16 * 16;
constexpr int kMiscOff = kRedOff + kMaxItems * kMegaConsumerWarps * 32 * 4;
constexpr int kGemvWorkEnd = kMiscOff + 16 * 4;

// Work-area layout for the attention phase: the K/V tile sits above every
// GEMV buffer, so the next tile can be fetched while the q|k|v phase still
// uses the GEMV view.
constexpr int kAttnRawOff = 0;                                          // bf16 [(G+2)*128]
constexpr int kAttnQOff = kAttnRawOff + (kMaxGroupHeads + 2) * kHD * 2;  // f32 [G][kQPitchM]
constexpr int kAttnKnOff = kAttnQOff + kMaxGroupHeads * kQPitchM * 4;   // f32 [128]
constexpr int kAttnVnOff = kAttnKnOff + kHD * 4;                        // f32 [128]
constexpr int kAttnScOff = kAttnVnOff + kHD * 4;                        // f32 [tile][G]
constexpr int kAttnStatOff = kAttnScOff + kAttnTileM * kMaxGroupHeads * 4;  // f32 [3][G]
// q|k|v partials of the KV head, [split][(G+2)*128] f32, staged by cp.async
// before raw is formed (q_s and the rest are written only afterwards)
constexpr int kAttnPartOff = kAttnQOff;
constexpr int kAttnPartEnd = kAttnPartOff + kMaxPartSplit * (kMaxGroupHeads + 2) * kHD * 4;
constexpr int kAttnTileOff =
    ((kGemvWorkEnd > kAttnPartEnd ? kGemvWorkEnd : kAttnPartEnd) + 127) / 128 * 128;
constexpr int kAttnVtOff = kAttnTileOff + kAttnTileM * kKPitchM * 2;    // bf16 V [tile][128]
constexpr int kAttnEnd = kAttnVtOff + kAttnTileM * kHD * 2;
// RMSNorm staging: the residual's partials [split][hidden] f32, by cp.async,
// over the tile buffers (no tile is in flight while a RMSNorm stages)
constexpr int kNormPartOff = kAttnTileOff;
constexpr int kNormPartEnd = kNormPartOff + kMaxPartSplit * 2048 * 4;
static_assert(kAttnStatOff + 3 * kMaxGroupHeads * 4 <= kAttnTileOff, "attention view");
static_assert(kAttnEnd <= kWorkBytes && kNormPartEnd <= kWorkBytes, "work area");
static_assert(kNC == 2 * kHD, "attention P.V: two threads per dimension");
static_assert((kAttnTileOff & 15) == 0 && (kAttnVtOff & 15) == 0, "cp.async destinations");

__device__ __forceinline__ void report(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ bool aborted(const int* flag) {
  return *reinterpret_cast<const volatile int*>(flag) != 0;
}
__device__ __forceinline__ void set_abort(int* flag) {
  *reinterpret_cast<volatile int*>(flag) = 1;
}

// Grid barrier over kBarCounters counters (CTA c arrives on counter c % 8,
// so arrivals do not serialise on one address), in two halves so that a CTA
// can issue the next phase's independent loads in between. `phases` =
// barriers passed so far including this one. Bounded wait: on expiry the
// error word and the CTA's abort flag are set and every consumer thread gets
// false (the step is abandoned; the flag also stops the producer).
__device__ void grid_arrive(const MegaParams& p, int* abort_flag) {
  consumers_sync();  // the phase's stores are done
  if (threadIdx.x == (int)(blockIdx.x % kBarCounters) && !aborted(abort_flag))
    red_release_add(p.bar + 32 * (blockIdx.x % kBarCounters), 1u);
}

__device__ bool grid_wait(const MegaParams& p, unsigned phases, int* abort_flag) {
  if (threadIdx.x < kBarCounters && !aborted(abort_flag)) {
    const int i = threadIdx.x;
    // CTAs on counter i: ceil((G - i) / 8)
    const unsigned target = phases * ((gridDim.x - i + kBarCounters - 1) / kBarCounters);
    const unsigned* c = p.bar + 32 * i;
    if (ld_acquire_u32(c) < target) {
      const unsigned long long t0 = globaltimer_ns();
      while (ld_acquire_u32(c) < target) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          report(p.err, kErrBarrier);
          set_abort(abort_flag);
          break;
        }
      }
    }
  }
  consumers_sync();
  return !aborted(abort_flag);
}

// ----------------------------------------------------------------- staging

// Norm weight slice a thread stages (loaded before the grid barrier).
__device__ __forceinline__ uint4 load_norm(const uint16_t* w, int H) {
  return threadIdx.x < H / 8 ? __ldg(reinterpret_cast<const uint4*>(w) + threadIdx.x)
                             : make_uint4(0u, 0u, 0u, 0u);
}

// Permutes one packed row's 8 activations into the MMA k order (x0,x4)
// (x1,x5) (x2,x6) (x3,x7), stores it at row r of xs and returns its beta
// share (the bf16 unpack offset 136 times the row's sum).
__device__ __forceinline__ float put_row(uint8_t* xs, int r, uint4 v) {
  uint4 o;
  o.x = __byte_perm(v.x, v.z, 0x5410);
  o.y = __byte_perm(v.x, v.z, 0x7632);
  o.z = __byte_perm(v.y, v.w, 0x5410);
  o.w = __byte_perm(v.y, v.w, 0x7632);
  *reinterpret_cast<uint4*>(xs + r * 16) = o;
  const uint32_t* oi = reinterpret_cast<const uint32_t*>(&o);
  const float ax = bfm(oi[0] & 0xffffu), ay = bfm(oi[0] >> 16);
  const float bx = bfm(oi[1] & 0xffffu), by = bfm(oi[1] >> 16);
  const float cx = bfm(oi[2] & 0xffffu), cy = bfm(oi[2] >> 16);
  const float dx = bfm(oi[3] & 0xffffu), dy = bfm(oi[3] >> 16);
  return kBF16Offset * (((ax + ay) + (cx + cy)) + ((bx + by) + (dx + dy)));
}

// Sums the beta shares of 16 consecutive rows (16 consecutive lanes) and
// stores the group's beta. Every lane of the warp must call it.
__device__ __forceinline__ void put_beta(float* beta, int r, bool active, float b) {
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) b += __shfl_xor_sync(0xffffffffu, b, off);
  if (active && (r & 15) == 0) beta[r >> 4] = b;
}

// h_new (one bf16 row of `hidden`) from the phase's source and its RMSNorm
// with the weight slice wv. Thread t owns elements 8t..8t+7, which is packed
// row t, so it stages groups [gk0, gk1) of x straight into xs (MMA k order,
// with beta) and, with to_xsrc, the whole row into xsrc. CTA 0 stores h_new
// to h_out.
__device__ void stage_rmsnorm(const MegaParams& p, int src, int64_t tok, const uint16_t* h_in,
                              const float* part, int split, uint4 wv, uint16_t* h_out, int gk0,
                              int gk1, bool to_xsrc, uint8_t* work) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int H = p.hidden;
  uint16_t* xsrc = reinterpret_cast<uint16_t*>(work + kXsrcOff);
  uint8_t* xs = work + kXsOff;
  float* beta = reinterpret_cast<float*>(work + kBetaOff);
  float* misc = reinterpret_cast<float*>(work + kMiscOff);
  float hv[8];
  float ss = 0.f;
  const bool act = t < H / 8;
  if (src != kSrcEmbed) {  // every partial of the row in flight at once (one round trip)
    float* ps = reinterpret_cast<float*>(work + kNormPartOff);
    for (int c = t; c < split * H / 4; c += kNC) cp_async16(ps + 4 * c, part + 4 * c);
    cp_async_commit();
    cp_async_wait_all();
    consumers_sync();
  }
  if (act) {
    if (src == kSrcEmbed) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(p.embed + (size_t)tok * H) + t);
      const uint32_t* vi = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        hv[2 * i] = bfm(vi[i] & 0xffffu);
        hv[2 * i + 1] = bfm(vi[i] >> 16);
      }
    } else {
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>(h_in) + t);
      const uint32_t* vi = reinterpret_cast<const uint32_t*>(&v);
      const float* ps = reinterpret_cast<const float*>(work + kNormPartOff);
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
      for (int s = 0; s < split; ++s) {  // staged in shared memory, summed in split order
        const float4 a = *reinterpret_cast<const float4*>(ps + (size_t)s * H + 8 * t);
        const float4 b = *reinterpret_cast<const float4*>(ps + (size_t)s * H + 8 * t + 4);
        acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
        acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        hv[2 * i] = rbfm(bfm(vi[i] & 0xffffu) + rbfm(acc[2 * i]));
        hv[2 * i + 1] = rbfm(bfm(vi[i] >> 16) + rbfm(acc[2 * i + 1]));
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(hv[i], hv[i], ss);
    if (h_out != nullptr && blockIdx.x == 0) {
      uint4 o;
      uint32_t* oi = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        oi[i] = (uint32_t)to_bfm(hv[2 * i]) | ((uint32_t)to_bfm(hv[2 * i + 1]) << 16);
      reinterpret_cast<uint4*>(h_out)[t] = o;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if (lane == 0) misc[warp] = ss;
  consumers_sync();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kMegaConsumerWarps; ++i) tot += misc[i];
  const float inv = rsqrtf(tot / (float)H + p.eps);
  uint4 x = make_uint4(0u, 0u, 0u, 0u);
  if (act) {
    const uint32_t* wi = reinterpret_cast<const uint32_t*>(&wv);
    uint32_t* xi = reinterpret_cast<uint32_t*>(&x);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a = rbfm(hv[2 * i] * inv) * bfm(wi[i] & 0xffffu);
      const float b = rbfm(hv[2 * i + 1] * inv) * bfm(wi[i] >> 16);
      xi[i] = (uint32_t)to_bfm(a) | ((uint32_t)to_bfm(b) << 16);
    }
    if (to_xsrc) reinterpret_cast<uint4*>(xsrc)[t] = x;
  }
  if (gk1 > gk0) {  // uniform over the CTA
    const int r = t - gk0 * 16;  // packed row t in the staged range
    const bool in = act && r >= 0 && r < (gk1 - gk0) * 16;
    const float b = in ? put_row(xs, r, x) : 0.f;
    put_beta(beta, r, in, b);
  }
  consumers_sync();  // xs, beta (and xsrc) complete; misc free again
}

// Position splits in use at this position: one per attention tile of cached
// positions, at most attn_splits (the attention and the merge both derive it
// from pos).
__device__ __forceinline__ int attn_splits_at(const MegaParams& p, int pos) {
  return max(1, min(p.attn_splits, (pos + 1 + kAttnTileM - 1) / kAttnTileM));
}

// Merged attention output for heads [hb, he) into xsrc (absolute index).
// A warp merges one (head, 64 dimensions): lanes 0..15 hold the splits'
// running maxima, lanes 16..31 their sums; the weights are broadcast by
// shuffles and every split's slice is read once, coalesced. Fixed order.
__device__ void stage_attn_merge(const MegaParams& p, int hb, int he, int pos, uint8_t* work) {
  const int G = p.group, A = attn_splits_at(p, pos);
  const int stride = G * (2 + kHD);  // floats per (kv head, split) record
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint16_t* xsrc = reinterpret_cast<uint16_t*>(work + kXsrcOff);
  for (int u = warp; u < (he - hb) * 2; u += kMegaConsumerWarps) {
    const int h = hb + (u >> 1), d0 = (u & 1) * 64;
    const int kvh = h / G, i = h - kvh * G;
    const float* rec = p.pattn + (size_t)kvh * p.attn_splits * stride;
    const int a_ml = lane & 15;
    float ml = (lane < 16) ? -INFINITY : 0.f;
    if (a_ml < A) ml = __ldcg(rec + (size_t)a_ml * stride + (lane < 16 ? i : G + i));
    float o0[kMaxAttnSplits], o1[kMaxAttnSplits];
#pragma unroll
    for (int a = 0; a < kMaxAttnSplits; ++a) {
      if (a < A) {
        const float* r = rec + (size_t)a * stride + 2 * G + i * kHD + d0 + lane;
        o0[a] = __ldcg(r);
        o1[a] = __ldcg(r + 32);
      }
    }
    float M = lane < 16 ? ml : -INFINITY;
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    M = __shfl_sync(0xffffffffu, M, 0);
    const float lsum = __shfl_sync(0xffffffffu, ml, (lane & 15) + 16);  // l of split lane&15
    const float w = (lane < 16 && a_ml < A && ml != -INFINITY) ? __expf(ml - M) : 0.f;
    float L = w * lsum;
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
    L = __shfl_sync(0xffffffffu, L, 0);
    float O0 = 0.f, O1 = 0.f;
#pragma unroll
    for (int a = 0; a < kMaxAttnSplits; ++a) {
      if (a < A) {
        const float wa = __shfl_sync(0xffffffffu, w, a);
        O0 = fmaf(wa, o0[a], O0);
        O1 = fmaf(wa, o1[a], O1);
      }
    }
    xsrc[h * kHD + d0 + lane] = to_bfm(O0 / L);
    xsrc[h * kHD + d0 + 32 + lane] = to_bfm(O1 / L);
  }
  consumers_sync();
}

// Stages groups [gk0, gk1) of x into xs in the MMA k order, with beta per
// group. kind: 0 = from xsrc (absolute k), 1 = SwiGLU of the gate|up partials.
__device__ void stage_x(const MegaParams& p, int kind, int gk0, int gk1, uint8_t* work) {
  const int t = threadIdx.x;
  const uint16_t* xsrc = reinterpret_cast<const uint16_t*>(work + kXsrcOff);
  uint8_t* xs = work + kXsOff;
  float* beta = reinterpret_cast<float*>(work + kBetaOff);
  const int rb = gk0 * 16, nrows = (gk1 - gk0) * 16;
  const float* pgu = p.part[2];
  const int I = p.inter;
  static_assert(kMaxStagedGroups * 16 <= 2 * kNC, "at most two staged rows per thread");
  // gate|up runs unsplit (planned with split 1), so a row's gate and up are
  // one partial each; both rows' loads are in flight together
  float4 gl[2][2], ul[2][2];
  if (kind == 1) {
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int r = u * kNC + t;
      const int k = (rb + min(r, nrows - 1)) * 8;
      if (r < nrows) {
        gl[u][0] = __ldcg(reinterpret_cast<const float4*>(pgu + k));
        gl[u][1] = __ldcg(reinterpret_cast<const float4*>(pgu + k) + 1);
        ul[u][0] = __ldcg(reinterpret_cast<const float4*>(pgu + I + k));
        ul[u][1] = __ldcg(reinterpret_cast<const float4*>(pgu + I + k) + 1);
      }
    }
  }
#pragma unroll
  for (int u = 0; u < 2; ++u) {  // uniform trip count
    const int base = u * kNC;
    if (base >= nrows) break;    // uniform over the CTA
    const int r = base + t;
    const bool active = r < nrows;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (active) {
      const int k = (rb + r) * 8;
      if (kind == 0) {
        v = *reinterpret_cast<const uint4*>(xsrc + k);
      } else {
        const float g[8] = {gl[u][0].x, gl[u][0].y, gl[u][0].z, gl[u][0].w,
                            gl[u][1].x, gl[u][1].y, gl[u][1].z, gl[u][1].w};
        const float uu[8] = {ul[u][0].x, ul[u][0].y, ul[u][0].z, ul[u][0].w,
                             ul[u][1].x, ul[u][1].y, ul[u][1].z, ul[u][1].w};
        uint32_t* vi = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float a = swiglu(rbfm(g[2 * i]), rbfm(uu[2 * i]));
          const float b = swiglu(rbfm(g[2 * i + 1]), rbfm(uu[2 * i + 1]));
          vi[i] = (uint32_t)to_bfm(a) | ((uint32_t)to_bfm(b) << 16);
        }
      }
    }
    const float b = active ? put_row(xs, r, v) : 0.f;
    put_beta(beta, r, active, b);
  }
  consumers_sync();
}

// ----------------------------------------------------------------- items

struct Ring {
  int slot = 0;
  uint32_t phase = 0;
  __device__ void advance() {
    if (++slot == kSlots) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

// Number of GEMV items of this CTA (items blockIdx.x, + gridDim.x, ...).
__device__ __forceinline__ int my_items(const MegaGemv& G) {
  return (int)blockIdx.x < G.items ? (G.items - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x
                                   : 0;
}

// Consumes this CTA's items of GEMV `gi` (x already staged for groups
// starting at gx0). The groups of all the CTA's stages are dealt to the warps
// round-robin; a warp keeps one accumulator per item and leaves it in `red`,
// and one barrier at the end precedes the fixed-order sum over warps. A failed
// wait sets the abort flag; every thread still runs the same barriers.
__device__ void gemv_items(const MegaParams& p, int gi, const MegaSmem& sm, Ring& ring, int gx0) {
  const MegaGemv& G = p.g[gi];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  uint8_t* work = sm.work;
  const float* beta = reinterpret_cast<const float*>(work + kBetaOff);
  float* red = reinterpret_cast<float*>(work + kRedOff);
  const uint32_t xs_base = smem_u32(work + kXsOff) + 2 * t * 16;
  const int ni = my_items(G);
  int task = 0;
  for (int k = 0; k < ni; ++k) {
    const int it = blockIdx.x + k * gridDim.x;
    const int strip = it / G.split, s = it - strip * G.split;
    const int g0 = s * G.gps, g1 = min(G.groups, g0 + G.gps);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};  // columns 4g .. 4g+3 (batch row 0)
    for (int sg = g0; sg < g1; sg += G.bg) {
      const int n = min(G.bg, g1 - sg);
      if (!aborted(sm.abort_flag) && !mbar_wait(&sm.full[ring.slot], ring.phase)) {
        report(p.err, kErrFullWait);
        set_abort(sm.abort_flag);
      }
      const bool live = !aborted(sm.abort_flag);
      const uint32_t wslot = smem_u32(sm.w) + ring.slot * kSlotBytes;
      const uint32_t sslot = smem_u32(sm.sc) + ring.slot * kSlotScaleBytes;
      // first group of this stage for this warp under the round-robin deal;
      // a warp's two groups of a stage (q, q + 8) run interleaved
      for (int q = (warp - task % kMegaConsumerWarps + kMegaConsumerWarps) % kMegaConsumerWarps;
           q < n && live; q += 2 * kMegaConsumerWarps) {
        const bool two = q + kMegaConsumerWarps < n;
        const int qb = two ? q + kMegaConsumerWarps : q;  // single: the second lane set is a copy
        const int ga = sg + q - gx0, gb = sg + qb - gx0;  // group indices in the staged x
        float ca[2][4], cb[2][4];
        {
          const float na = -beta[ga], nb = -beta[gb];
#pragma unroll
          for (int z = 0; z < 2; ++z)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              ca[z][i] = na;
              cb[z][i] = nb;
            }
        }
        const uint32_t wa_box = wslot + q * kGroupBytes, wb_box = wslot + qb * kGroupBytes;
#pragma unroll
        for (int o = 0; o < 2; ++o) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int row = 8 * o + 2 * t + e;
            const uint32_t woff = row * 128 + ((g ^ (2 * t + e)) << 4);
            const uint4 wa = lds128(wa_box + woff);
            const uint4 wb = lds128(wb_box + woff);
            const uint4 xa = lds128(xs_base + (ga * 16 + 8 * o + e) * 16);
            const uint4 xb = lds128(xs_base + (gb * 16 + 8 * o + e) * 16);
            uint32_t h0[4], h1[4], k0[4], k1[4];
            unpack_nibbles<true>(wa.x, h0);
            unpack_nibbles<true>(wa.y, h1);
            unpack_nibbles<true>(wb.x, k0);
            unpack_nibbles<true>(wb.y, k1);
            mma_16816<true>(ca[0], h0[0], h1[0], h0[1], h1[1], xa.x, xa.y);
            mma_16816<true>(cb[0], k0[0], k1[0], k0[1], k1[1], xb.x, xb.y);
            mma_16816<true>(ca[0], h0[2], h1[2], h0[3], h1[3], xa.z, xa.w);
            mma_16816<true>(cb[0], k0[2], k1[2], k0[3], k1[3], xb.z, xb.w);
            unpack_nibbles<true>(wa.z, h0);
            unpack_nibbles<true>(wa.w, h1);
            unpack_nibbles<true>(wb.z, k0);
            unpack_nibbles<true>(wb.w, k1);
            mma_16816<true>(ca[1], h0[0], h1[0], h0[1], h1[1], xa.x, xa.y);
            mma_16816<true>(cb[1], k0[0], k1[0], k0[1], k1[1], xb.x, xb.y);
            mma_16816<true>(ca[1], h0[2], h1[2], h0[3], h1[3], xa.z, xa.w);
            mma_16816<true>(cb[1], k0[2], k1[2], k0[3], k1[3], xb.z, xb.w);
          }
        }
        const uint32_t sa = sslot + q * kScaleGroupBytes + 4 * g * 2;
        const uint32_t sb = sslot + qb * kScaleGroupBytes + 4 * g * 2;
        const uint32_t a01 = lds32(sa), a23 = lds32(sa + 4);
        const float2 fa01 = __half22float2(*reinterpret_cast<const __half2*>(&a01));
        const float2 fa23 = __half22float2(*reinterpret_cast<const __half2*>(&a23));
        acc[0] = fmaf(fa01.x, ca[0][0], acc[0]);
        acc[1] = fmaf(fa01.y, ca[0][2], acc[1]);
        acc[2] = fmaf(fa23.x, ca[1][0], acc[2]);
        acc[3] = fmaf(fa23.y, ca[1][2], acc[3]);
        if (two) {
          const uint32_t b01 = lds32(sb), b23 = lds32(sb + 4);
          const float2 fb01 = __half22float2(*reinterpret_cast<const __half2*>(&b01));
          const float2 fb23 = __half22float2(*reinterpret_cast<const __half2*>(&b23));
          acc[0] = fmaf(fb01.x, cb[0][0], acc[0]);
          acc[1] = fmaf(fb01.y, cb[0][2], acc[1]);
          acc[2] = fmaf(fb23.x, cb[1][0], acc[2]);
          acc[3] = fmaf(fb23.y, cb[1][2], acc[3]);
        }
      }
      task += n;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty[ring.slot]);
      ring.advance();
    }
    if (t == 0) {  // this warp's share of item k (zeros if it had no group)
      float* r = red + (k * kMegaConsumerWarps + warp) * 32 + 4 * g;
      r[0] = acc[0];
      r[1] = acc[1];
      r[2] = acc[2];
      r[3] = acc[3];
    }
  }
  consumers_sync();
  float* out = p.part[gi];
  for (int idx = threadIdx.x; idx < ni * 32; idx += kNC) {
    const int k = idx >> 5, col = idx & 31;
    const int it = blockIdx.x + k * gridDim.x;
    const int strip = it / G.split, s = it - strip * G.split;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kMegaConsumerWarps; ++w) v += red[(k * kMegaConsumerWarps + w) * 32 + col];
    out[(size_t)s * G.N + strip * 32 + col] = v;
  }
  // red is read above and rewritten only after the next grid barrier
}

// The CTA's range of K groups for GEMV gi (all its items share it).
__device__ __forceinline__ bool item_range(const MegaGemv& G, int* gk0, int* gk1) {
  if ((int)blockIdx.x >= G.items) return false;
  if (G.split == 1) {
    *gk0 = 0;
    *gk1 = G.groups;
  } else {
    const int s = blockIdx.x % G.split;
    *gk0 = s * G.gps;
    *gk1 = min(G.groups, *gk0 + G.gps);
  }
  return true;
}

// ----------------------------------------------------------------- attention

__device__ __forceinline__ float rope_m(const uint16_t* head, int d, float c, float s) {
  const float x = bfm(head[d]);
  const float partner = bfm(head[d ^ 64]);
  const float rot = (d < 64) ? -partner : partner;
  return rbfm(rbfm(x * c) + rbfm(rot * s));
}

// What the attention phase of a CTA reads that the q|k|v phase does not
// write: the positions of its split, RoPE factors and bias in registers, and
// the first K/V tile (asynchronous copies into the tile buffers).
struct AttnPre {
  int kvh, a, j0, j1;
  float c, s;                     // RoPE factors of dimension threadIdx.x (< 128)
  float bias[5];                  // q|k|v bias of the elements this thread loads
};

__device__ __forceinline__ int attn_elem(const MegaParams& p, int kvh, int i) {
  const int G = p.group, H = p.hidden;
  const int h = i / kHD, d = i - h * kHD;
  return h < G ? (kvh * G + h) * kHD + d
               : (h == G ? H + kvh * kHD + d : H + p.kv_heads * kHD + kvh * kHD + d);
}

__device__ void load_kv_tile(const MegaParams& p, size_t cache_head, int t0, int nc,
                             uint8_t* work) {
  uint16_t* kt = reinterpret_cast<uint16_t*>(work + kAttnTileOff);
  uint16_t* vt = reinterpret_cast<uint16_t*>(work + kAttnVtOff);
  const uint16_t* kc = p.k_cache + cache_head * kHD;
  const uint16_t* vc = p.v_cache + cache_head * kHD;
  for (int i = threadIdx.x; i < nc * 16; i += kNC) {
    const int r = i >> 4, cc = i & 15;
    cp_async16(kt + r * kKPitchM + 8 * cc, kc + (size_t)(t0 + r) * kHD + 8 * cc);
    cp_async16(vt + r * kHD + 8 * cc, vc + (size_t)(t0 + r) * kHD + 8 * cc);
  }
  cp_async_commit();
}

__device__ AttnPre attention_prefetch(const MegaParams& p, int l, int pos, uint8_t* work) {
  AttnPre pre;
  const int A = attn_splits_at(p, pos);
  pre.kvh = blockIdx.x / A;
  pre.a = blockIdx.x - pre.kvh * A;
  const int P = pos + 1;
  const int chunk = (P + A - 1) / A;
  pre.j0 = min(P, pre.a * chunk);
  pre.j1 = min(P, pre.j0 + chunk);
  const int t = threadIdx.x;
  pre.c = pre.s = 0.f;
  if (t < kHD) {
    pre.c = bfm(__ldg(p.cos_t + (size_t)pos * kHD + t));
    pre.s = bfm(__ldg(p.sin_t + (size_t)pos * kHD + t));
  }
  const int nq = p.g[0].N;
  const uint16_t* bias = p.qkv_bias + (size_t)l * nq;
#pragma unroll
  for (int j = 0; j < 5; ++j) {
    const int i = t + j * kNC;
    pre.bias[j] = i < (p.group + 2) * kHD ? bfm(__ldg(bias + attn_elem(p, pre.kvh, i))) : 0.f;
  }
  const size_t cache_head = ((size_t)l * p.kv_heads + pre.kvh) * p.max_seq;
  const int t1 = min(pre.j1, pre.j0 + kAttnTileM);
  const int nc = max(0, min(t1, pos) - pre.j0);  // rows already in the cache
  load_kv_tile(p, cache_head, pre.j0, nc, work);
  return pre;
}

__device__ void attention_phase(const MegaParams& p, int l, int pos, const AttnPre& pre,
                                uint8_t* work) {
  const int G = p.group, A = p.attn_splits;  // record stride: the planned split count
  const int kvh = pre.kvh, a = pre.a, j0 = pre.j0, j1 = pre.j1;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  uint16_t* raw = reinterpret_cast<uint16_t*>(work + kAttnRawOff);
  float* q_s = reinterpret_cast<float*>(work + kAttnQOff);
  float* kn_s = reinterpret_cast<float*>(work + kAttnKnOff);
  float* vn_s = reinterpret_cast<float*>(work + kAttnVnOff);
  float* sc_s = reinterpret_cast<float*>(work + kAttnScOff);
  float* hm_s = reinterpret_cast<float*>(work + kAttnStatOff);
  float* hl_s = hm_s + kMaxGroupHeads;
  float* ha_s = hl_s + kMaxGroupHeads;
  const uint16_t* kt_s = reinterpret_cast<const uint16_t*>(work + kAttnTileOff);
  const uint16_t* vt_s = reinterpret_cast<const uint16_t*>(work + kAttnVtOff);
  const int nq = p.g[0].N;
  const MegaGemv& gq = p.g[0];
  const float* pq = p.part[0];
  // q heads, k and v of this KV head: bf16(sum of partials + bias)
  {  // every split's q heads, k and v of this KV head in flight at once (cp.async)
    float* ps = reinterpret_cast<float*>(work + kAttnPartOff);
    const int per = (G + 2) * kHD;  // floats per split; 16-byte chunks never cross a head
    for (int c = t; c < gq.split * per / 4; c += kNC) {
      const int s = (4 * c) / per, i = 4 * c - s * per;
      cp_async16(ps + 4 * c, pq + (size_t)s * nq + attn_elem(p, kvh, i));
    }
    cp_async_commit();
    cp_async_wait_all();
    consumers_sync();
#pragma unroll
    for (int j = 0; j < 5; ++j) {
      const int i = t + j * kNC;
      if (i < per) {
        float v = 0.f;
        for (int s = 0; s < gq.split; ++s) v += ps[s * per + i];
        raw[i] = to_bfm(v + pre.bias[j]);
      }
    }
  }
  const size_t cache_head = ((size_t)l * p.kv_heads + kvh) * p.max_seq;
  if (t < G) {
    hm_s[t] = -INFINITY;
    hl_s[t] = 0.f;
  }
  consumers_sync();
  if (t < kHD) {
    for (int h = 0; h < G; ++h) q_s[h * kQPitchM + t] = rope_m(raw + h * kHD, t, pre.c, pre.s);
    const float kr = rope_m(raw + G * kHD, t, pre.c, pre.s);
    const float vv = bfm(raw[(G + 1) * kHD + t]);
    kn_s[t] = kr;
    vn_s[t] = vv;
    if (pos >= j0 && pos < j1) {  // this split owns the new position
      p.k_cache[(cache_head + pos) * kHD + t] = to_bfm(kr);
      p.v_cache[(cache_head + pos) * kHD + t] = to_bfm(vv);
    }
  }
  const int dd = t & (kHD - 1), hh = t >> 7;  // P.V: dimension and head parity
  float o[kMaxGroupHeads / 2];
#pragma unroll
  for (int j = 0; j < kMaxGroupHeads / 2; ++j) o[j] = 0.f;
  for (int t0 = j0; t0 < j1; t0 += kAttnTileM) {
    const int t1 = min(j1, t0 + kAttnTileM);
    const int n = t1 - t0;
    if (t0 != j0) {  // later tiles: the previous one is consumed
      consumers_sync();
      load_kv_tile(p, cache_head, t0, max(0, min(t1, pos) - t0), work);
    }
    cp_async_wait_all();
    consumers_sync();  // tile, q_s and kn_s visible to every consumer
    // scores: four consecutive lanes share one (position, head) dot product,
    // lane part p taking the words 4w + p, then a fixed two-step shuffle sum
    for (int base = 0; base < n * G * 4; base += kNC) {  // uniform trip count
      const int i = base + t;
      const int pi = i >> 2, part = i & 3;
      const bool act = pi < n * G;
      float d = 0.f;
      if (act) {
        const int jl = pi / G, h = pi - jl * G;
        const float* qh = q_s + h * kQPitchM;
        if (t0 + jl == pos) {
#pragma unroll 4
          for (int w = 0; w < kHD / 8; ++w) {
            const int e = 2 * (4 * w + part);
            d = fmaf(qh[e], kn_s[e], d);
            d = fmaf(qh[e + 1], kn_s[e + 1], d);
          }
        } else {
          const uint32_t* kw = reinterpret_cast<const uint32_t*>(kt_s + jl * kKPitchM);
#pragma unroll 4
          for (int w = 0; w < kHD / 8; ++w) {
            const uint32_t kk = kw[4 * w + part];
            const int e = 2 * (4 * w + part);
            d = fmaf(qh[e], bfm(kk & 0xffffu), d);
            d = fmaf(qh[e + 1], bfm(kk >> 16), d);
          }
        }
      }
      d += __shfl_xor_sync(0xffffffffu, d, 1);
      d += __shfl_xor_sync(0xffffffffu, d, 2);
      if (act && part == 0) sc_s[pi] = d * p.scale;
    }
    consumers_sync();
    for (int h = warp; h < G; h += kMegaConsumerWarps) {  // online softmax per head
      float mx = -INFINITY;
      for (int jl = lane; jl < n; jl += 32) mx = fmaxf(mx, sc_s[jl * G + h]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_old = hm_s[h];
      const float m_new = fmaxf(m_old, mx);
      float sum = 0.f;
      for (int jl = lane; jl < n; jl += 32) {
        const float pr = __expf(sc_s[jl * G + h] - m_new);
        sc_s[jl * G + h] = pr;
        sum += pr;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      if (lane == 0) {
        const float alpha = (m_old == -INFINITY) ? 0.f : __expf(m_old - m_new);
        ha_s[h] = alpha;
        hl_s[h] = hl_s[h] * alpha + sum;
        hm_s[h] = m_new;
      }
    }
    consumers_sync();
    {  // P.V: thread t owns dimension t & 127 of the heads h = (t >> 7) + 2j
#pragma unroll
      for (int j = 0; j < kMaxGroupHeads / 2; ++j)
        if (hh + 2 * j < G) o[j] *= ha_s[hh + 2 * j];
      for (int jl = 0; jl < n; ++jl) {
        const float vj = (t0 + jl == pos) ? vn_s[dd] : bfm(vt_s[jl * kHD + dd]);
#pragma unroll
        for (int j = 0; j < kMaxGroupHeads / 2; ++j)
          if (hh + 2 * j < G) o[j] = fmaf(sc_s[jl * G + hh + 2 * j], vj, o[j]);
      }
    }
  }
  cp_async_wait_all();  // an empty split still committed an (empty) group
  consumers_sync();
  // this split's partial record (an empty split leaves m = -inf, l = 0, o = 0)
  float* rec = p.pattn + ((size_t)kvh * A + a) * G * (2 + kHD);
  if (t < G) {
    rec[t] = hm_s[t];
    rec[G + t] = hl_s[t];
  }
#pragma unroll
  for (int j = 0; j < kMaxGroupHeads / 2; ++j)
    if (hh + 2 * j < G) rec[2 * G + (hh + 2 * j) * kHD + dd] = o[j];
}

// ----------------------------------------------------------------- lm_head

template <int CH>
__device__ void lm_phase(const MegaParams& p, const MegaSmem& sm, Ring& ring,
                         unsigned long long* best_out) {
  constexpr int H = CH * 256;
  constexpr uint32_t kRowBytes = H * 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint16_t* xsrc = reinterpret_cast<const uint16_t*>(sm.work + kXsrcOff);
  float xr[CH][8];
#pragma unroll
  for (int c = 0; c < CH; ++c)
#pragma unroll
    for (int i = 0; i < 8; ++i) xr[c][i] = bfm(xsrc[8 * (32 * c + lane) + i]);
  const int per = (p.vocab + gridDim.x - 1) / gridDim.x;
  const int r0 = min(p.vocab, (int)blockIdx.x * per), r1 = min(p.vocab, r0 + per);
  unsigned long long best = 0;
  for (int rs = r0; rs < r1; rs += p.lm_rows) {
    const int nrows = min(p.lm_rows, r1 - rs);
    if (!aborted(sm.abort_flag) && !mbar_wait(&sm.full[ring.slot], ring.phase)) {
      report(p.err, kErrFullWait);
      set_abort(sm.abort_flag);
    }
    if (warp < nrows && !aborted(sm.abort_flag)) {
      const uint4* ra =
          reinterpret_cast<const uint4*>(sm.w + (size_t)ring.slot * kSlotBytes + warp * kRowBytes);
      float da = 0.f;
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const uint4 a = ra[32 * c + lane];
        const uint32_t* av = reinterpret_cast<const uint32_t*>(&a);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          da = fmaf(bfm(av[i] & 0xffffu), xr[c][2 * i], da);
          da = fmaf(bfm(av[i] >> 16), xr[c][2 * i + 1], da);
        }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) da += __shfl_xor_sync(0xffffffffu, da, off);
      if (lane == 0) {
        const int ia = rs + warp;
        const uint16_t la = to_bfm(da);
        if (p.logits) p.logits[ia] = la;
        const unsigned long long ka =
            ((unsigned long long)order_key_m(bfm(la)) << 32) | (0xffffffffu - (uint32_t)ia);
        best = ka > best ? ka : best;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[ring.slot]);
    ring.advance();
  }
  *best_out = best;
}

// ----------------------------------------------------------------- producer

__device__ void producer(const MegaParams& p, const MegaSmem& sm, const MegaMaps& maps) {
  int issued = 0;
  Ring ring;
  bool ok = true;
  auto acquire = [&]() -> bool {
    if (aborted(sm.abort_flag)) return false;
    if (issued >= kSlots && !mbar_wait(&sm.empty[ring.slot], ring.phase ^ 1u)) {
      report(p.err, kErrEmptyWait);
      set_abort(sm.abort_flag);
      return false;
    }
    return true;
  };
  for (int l = 0; l < p.layers && ok; ++l) {
    for (int gi = 0; gi < 4 && ok; ++gi) {
      const MegaGemv& G = p.g[gi];
      const int row_base = l * (G.K / 8);
      const int grp_base = l * G.groups;
      for (int it = blockIdx.x; it < G.items && ok; it += gridDim.x) {
        const int strip = it / G.split, s = it - strip * G.split;
        const int g0 = s * G.gps, g1 = min(G.groups, g0 + G.gps);
        for (int sg = g0; sg < g1; sg += G.bg) {
          if (!acquire()) {
            ok = false;
            break;
          }
          uint64_t* fb = &sm.full[ring.slot];
          uint8_t* wd = sm.w + ring.slot * kSlotBytes;
          uint8_t* sd = sm.sc + ring.slot * kSlotScaleBytes;
          // 128B-swizzled boxes land on 1024-byte boundaries, plain boxes on 128
          if ((smem_u32(wd) & 1023u) || (smem_u32(sd) & 127u)) {
            report(p.err, kErrAlign);
            set_abort(sm.abort_flag);
            ok = false;
            break;
          }
          // whole boxes: the last stage of an item may also bring groups past
          // its range (unused; past the tensor's end they are zero-filled)
          mbar_arrive_expect_tx(fb, (uint32_t)G.bg * (kGroupBytes + kScaleGroupBytes));
          tma_load_2d(wd, &maps.w[gi], fb, strip * 32, row_base + sg * 16);
          tma_load_2d(sd, &maps.s[gi], fb, strip * 32, grp_base + sg);
          ++issued;
          ring.advance();
        }
      }
    }
  }
  if (ok) {  // lm_head rows of this CTA
    const uint32_t row_bytes = (uint32_t)p.hidden * 2;
    const int per = (p.vocab + gridDim.x - 1) / gridDim.x;
    const int r0 = min(p.vocab, (int)blockIdx.x * per), r1 = min(p.vocab, r0 + per);
    for (int rs = r0; rs < r1; rs += p.lm_rows) {
      const int nrows = min(p.lm_rows, r1 - rs);
      if (!acquire()) break;
      const uint32_t bytes = (uint32_t)nrows * row_bytes;
      if ((smem_u32(sm.w + ring.slot * kSlotBytes) & 15u) || (bytes & 15u)) {
        report(p.err, kErrAlign);
        set_abort(sm.abort_flag);
        break;
      }
      mbar_arrive_expect_tx(&sm.full[ring.slot], bytes);
      bulk_load_m(sm.w + ring.slot * kSlotBytes, p.embed + (size_t)rs * p.hidden, bytes,
                  &sm.full[ring.slot]);
      ++issued;
      ring.advance();
    }
  }
  // no copy into this CTA's shared memory may be left in flight
  for (int j = max(0, issued - kSlots); j < issued; ++j)
    if (!mbar_wait(&sm.full[j % kSlots], (j / kSlots) & 1)) report(p.err, kErrDrainWait);
}

}  // namespace

__global__ void __launch_bounds__(kMegaThreads, 1)
    decode_step_kernel(const __grid_constant__ MegaMaps maps, const __grid_constant__ MegaParams p) {
  extern __shared__ uint8_t smem_raw_m[];
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw_m) + 1023) & ~static_cast<uintptr_t>(1023));
  MegaSmem sm;
  sm.w = base;
  sm.sc = base + kSlots * kSlotBytes;
  sm.work = sm.sc + kSlots * kSlotScaleBytes;
  sm.full = reinterpret_cast<uint64_t*>(sm.work + kWorkBytes);
  sm.empty = sm.full + kSlots;
  sm.abort_flag = reinterpret_cast<int*>(sm.empty + kSlots);
  unsigned long long* s_best = reinterpret_cast<unsigned long long*>(sm.abort_flag + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kMegaConsumerWarps);
    }
    *sm.abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kMegaConsumerWarps) {
    if (lane == 0) {
      for (int i = 0; i < 4; ++i) {
        tma_prefetch_desc(&maps.w[i]);
        tma_prefetch_desc(&maps.s[i]);
      }
      producer(p, sm, maps);
    }
    return;
  }

  // ------------------------------------------------------------ consumers
  // The step state: read once (the last CTA advances it after everyone is done).
  const int64_t raw_pos = *p.pos;
  const int pos = raw_pos < 0 ? 0 : (raw_pos >= p.max_seq ? p.max_seq - 1 : (int)raw_pos);
  int64_t tok = (raw_pos < *p.prompt_len) ? p.prompt[pos] : *p.token;
  tok = tok < 0 ? 0 : (tok >= p.vocab ? p.vocab - 1 : tok);

  Ring ring;
  unsigned phases = 0;  // grid barriers passed
  bool ok = true;
  const int H = p.hidden;
  const bool attn_cta = (int)blockIdx.x < p.kv_heads * attn_splits_at(p, pos);
  uint4 wv = load_norm(p.in_norm, H);  // the next RMSNorm's weight slice
  for (int l = 0; l < p.layers; ++l) {
    int gk0 = 0, gk1 = 0;
    // ---- q|k|v: x = rmsnorm(h), h = embedding row or h1 + down partials
    {
      const bool mine = item_range(p.g[0], &gk0, &gk1);
      if (!mine) gk0 = gk1 = 0;
      if (mine || blockIdx.x == 0) {
        if (l == 0)
          stage_rmsnorm(p, kSrcEmbed, tok, nullptr, nullptr, 0, wv, p.h0, gk0, gk1, false,
                        sm.work);
        else
          stage_rmsnorm(p, kSrcH1Down, tok, p.h1, p.part[3], p.g[3].split, wv, p.h0, gk0, gk1,
                        false, sm.work);
      }
      if (mine) gemv_items(p, 0, sm, ring, gk0);
    }
    grid_arrive(p, sm.abort_flag);
    AttnPre pre{};
    if (attn_cta) pre = attention_prefetch(p, l, pos, sm.work);  // overlaps the barrier
    if (!(ok = grid_wait(p, ++phases, sm.abort_flag))) break;
    // ---- attention
    if (attn_cta) attention_phase(p, l, pos, pre, sm.work);
    grid_arrive(p, sm.abort_flag);
    if (!(ok = grid_wait(p, ++phases, sm.abort_flag))) break;
    // ---- o: x = merged attention (head_dim = 128: K group g is head g)
    if (item_range(p.g[1], &gk0, &gk1)) {
      stage_attn_merge(p, gk0, gk1, pos, sm.work);
      stage_x(p, 0, gk0, gk1, sm.work);
      gemv_items(p, 1, sm, ring, gk0);
    }
    grid_arrive(p, sm.abort_flag);
    wv = load_norm(p.post_norm + (size_t)l * H, H);
    if (!(ok = grid_wait(p, ++phases, sm.abort_flag))) break;
    // ---- gate|up: x = rmsnorm(h1), h1 = h0 + o partials
    {
      const bool mine = item_range(p.g[2], &gk0, &gk1);
      if (!mine) gk0 = gk1 = 0;
      if (mine || blockIdx.x == 0)
        stage_rmsnorm(p, kSrcH0O, tok, p.h0, p.part[1], p.g[1].split, wv, p.h1, gk0, gk1, false,
                      sm.work);
      if (mine) gemv_items(p, 2, sm, ring, gk0);
    }
    grid_arrive(p, sm.abort_flag);
    if (!(ok = grid_wait(p, ++phases, sm.abort_flag))) break;
    // ---- down: x = silu(gate) * up
    if (item_range(p.g[3], &gk0, &gk1)) {
      stage_x(p, 1, gk0, gk1, sm.work);
      gemv_items(p, 3, sm, ring, gk0);
    }
    grid_arrive(p, sm.abort_flag);
    wv = load_norm(l + 1 < p.layers ? p.in_norm + (size_t)(l + 1) * H : p.final_norm, H);
    if (!(ok = grid_wait(p, ++phases, sm.abort_flag))) break;
  }

  unsigned long long best = 0;
  if (ok) {
    // ---- lm_head: x = rmsnorm(h1 + down partials) with the final norm
    stage_rmsnorm(p, kSrcH1Down, tok, p.h1, p.part[3], p.g[3].split, wv, nullptr, 0, 0, true,
                  sm.work);
    switch (H / 256) {
      case 1: lm_phase<1>(p, sm, ring, &best); break;
      case 2: lm_phase<2>(p, sm, ring, &best); break;
      case 4: lm_phase<4>(p, sm, ring, &best); break;
      case 6: lm_phase<6>(p, sm, ring, &best); break;
      default: lm_phase<8>(p, sm, ring, &best); break;
    }
  }
  consumers_sync();
  if (aborted(sm.abort_flag)) return;  // uniform: read after the barrier
  if (lane == 0) s_best[warp] = best;
  consumers_sync();
  if (threadIdx.x == 0) {
    unsigned long long b = 0;
    for (int w = 0; w < kMegaConsumerWarps; ++w) b = s_best[w] > b ? s_best[w] : b;
    atomicMax(p.best, b);
    __threadfence();
    const unsigned ticket = atomicAdd(p.done, 1u);
    if (ticket == gridDim.x - 1) {  // last CTA: every other CTA's maximum is visible
      __threadfence();
      const unsigned long long fin = atomicAdd(p.best, 0ull);
      *p.token = (int64_t)(0xffffffffu - (uint32_t)(fin & 0xffffffffu));
      *p.pos = raw_pos + 1;
      *p.best = 0;  // leave the scratch counters zeroed for the next step
      *p.done = 0;
      for (int i = 0; i < kBarCounters; ++i) p.bar[32 * i] = 0;
      __threadfence();
    }
  }
}

// ----------------------------------------------------------------- host side

namespace {

struct MegaLayout {
  MegaGemv g[4];
  int attn_splits = 0;
  size_t off_h0 = 0, off_h1 = 0, off_part[4] = {0, 0, 0, 0}, off_attn = 0, total = 0;
};

MegaGemv plan_gemv(int N, int K, int ctas) {
  MegaGemv G;
  G.N = N;
  G.K = K;
  G.groups = K / 128;
  G.strips = N / 32;
  int split = 1;
  if (G.strips < ctas) split = std::min(std::min(G.groups, ctas / G.strips), kMaxPartSplit);
  split = std::max(split, (G.groups + kMaxStagedGroups - 1) / kMaxStagedGroups);  // x fits
  G.gps = (G.groups + split - 1) / split;
  G.split = (G.groups + G.gps - 1) / G.gps;  // no empty split
  G.items = G.strips * G.split;
  G.bg = std::min(kGroupsPerStage, G.gps);
  return G;
}

size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

bool plan_layout(const w4_decode_model& m, int ctas, MegaLayout* L) {
  const int nq = m.hidden + 2 * m.kv_heads * 128;
  L->g[0] = plan_gemv(nq, m.hidden, ctas);
  L->g[1] = plan_gemv(m.hidden, m.hidden, ctas);
  L->g[2] = plan_gemv(2 * m.intermediate, m.hidden, ctas);
  if (L->g[2].split != 1) {  // the SwiGLU staging reads one gate|up partial
    MegaGemv& G = L->g[2];
    G.split = 1;
    G.gps = G.groups;
    G.items = G.strips;
    G.bg = std::min(kGroupsPerStage, G.gps);
  }
  L->g[3] = plan_gemv(m.hidden, m.intermediate, ctas);
  for (int i = 0; i < 4; ++i) {
    if (L->g[i].split > 1 && L->g[i].items > ctas) return false;  // one item, one K range
    if (L->g[i].items > kMaxItems * ctas) return false;           // per-CTA accumulators
    if (L->g[i].gps > kMaxStagedGroups) return false;
    if (L->g[i].split > kMaxPartSplit) return false;
  }
  L->attn_splits = std::max(1, std::min(16, ctas / m.kv_heads));
  size_t off = 2048;  // barrier counters @0 (128 B apart), done @1024, best @1152
  L->off_h0 = off;
  off = align256(off + (size_t)m.hidden * 2);
  L->off_h1 = off;
  off = align256(off + (size_t)m.hidden * 2);
  for (int i = 0; i < 4; ++i) {
    L->off_part[i] = off;
    off = align256(off + (size_t)L->g[i].split * L->g[i].N * 4);
  }
  L->off_attn = off;
  const int G = m.heads / m.kv_heads;
  off = align256(off + (size_t)m.kv_heads * L->attn_splits * G * (2 + 128) * 4);
  L->total = off;
  return true;
}

size_t mega_smem_bytes() {
  return 1024 + (size_t)kSlots * (kSlotBytes + kSlotScaleBytes) + kWorkBytes + 256;  // + barriers
}

bool encode_map(CUtensorMap* map, CUtensorMapDataType dt, int elem, const void* base,
                uint64_t cols, uint64_t rows, uint32_t box_cols, uint32_t box_rows,
                CUtensorMapSwizzle swz) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * (uint64_t)elem};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int validate_model(const w4_decode_model& m) {
  if (m.layers < 1 || m.hidden <= 0 || m.intermediate <= 0 || m.heads <= 0 || m.kv_heads <= 0 ||
      m.vocab <= 0 || m.max_seq <= 0)
    return fail(W4_ERR_INVALID_ARG, "decode model: non-positive dimension");
  if (m.head_dim != 128) return fail(W4_ERR_UNSUPPORTED, "decode model: head_dim must be 128");
  if (m.heads * 128 != m.hidden)
    return fail(W4_ERR_INVALID_ARG, "decode model: heads * head_dim != hidden");
  if (m.heads % m.kv_heads || m.heads / m.kv_heads > kMaxGroupHeads)
    return fail(W4_ERR_UNSUPPORTED, "decode model: heads / kv_heads must divide and be <= %d",
                kMaxGroupHeads);
  const int H = m.hidden;
  if (!(H == 256 || H == 512 || H == 1024 || H == 1536 || H == 2048))
    return fail(W4_ERR_UNSUPPORTED, "decode model: hidden must be 256, 512, 1024, 1536 or 2048");
  if (m.intermediate % 128)
    return fail(W4_ERR_INVALID_ARG, "decode model: intermediate must be a multiple of 128");
  if ((long long)m.vocab * H * 2 > (1ll << 40))
    return fail(W4_ERR_UNSUPPORTED, "decode model: embedding too large");
  const void* ptrs[] = {m.qkv_packed, m.qkv_scales, m.o_packed,   m.o_scales,  m.gu_packed,
                        m.gu_scales,  m.down_packed, m.down_scales, m.qkv_bias, m.in_norm,
                        m.post_norm,  m.final_norm, m.embed,       m.cos_table, m.sin_table,
                        m.k_cache,    m.v_cache,    m.prompt,      m.prompt_len, m.token,
                        m.pos};
  for (const void* q : ptrs)
    if (q == nullptr) return fail(W4_ERR_INVALID_ARG, "decode model: null pointer");
  const void* a16[] = {m.qkv_packed, m.qkv_scales, m.o_packed,  m.o_scales, m.gu_packed,
                       m.gu_scales,  m.down_packed, m.down_scales, m.embed,   m.k_cache,
                       m.v_cache,    m.in_norm,    m.post_norm,  m.final_norm};
  for (const void* q : a16)
    if (reinterpret_cast<uintptr_t>(q) & 15)
      return fail(W4_ERR_ALIGNMENT, "decode model: weights, norms and caches need 16-byte alignment");
  return W4_OK;
}

int check_device(const DeviceInfo& di) {
  if (mega_smem_bytes() > (size_t)di.max_smem_optin)
    return fail(W4_ERR_UNSUPPORTED, "decode step needs %zu B of shared memory", mega_smem_bytes());
  return W4_OK;
}

}  // namespace

int mega_init_device(const DeviceInfo& di) {
  cudaError_t e = cudaFuncSetAttribute(decode_step_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)mega_smem_bytes());
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(decode step smem)");
  e = cudaFuncSetAttribute(decode_step_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(decode step carveout)");
  (void)di;
  return W4_OK;
}

int decode_step_scratch_bytes(const w4_decode_model& m, size_t* bytes) {
  int st = validate_model(m);  // before any CUDA call
  if (st != W4_OK) return st;
  int dev = 0;
  st = current_device(&dev);
  if (st != W4_OK) return st;
  const DeviceInfo& di = device_info(dev);
  st = check_device(di);
  if (st != W4_OK) return st;
  MegaLayout L;
  if (!plan_layout(m, di.sm_count, &L))
    return fail(W4_ERR_UNSUPPORTED, "decode model does not fit the step's work split");
  *bytes = L.total;
  return W4_OK;
}

int launch_decode_step(const w4_decode_model& m, void* scratch, size_t scratch_bytes,
                       cudaStream_t stream) {
  int st = validate_model(m);  // before any CUDA call
  if (st != W4_OK) return st;
  if (scratch == nullptr) return fail(W4_ERR_INVALID_ARG, "decode step: null scratch");
  int dev = 0;
  st = current_device(&dev);
  if (st != W4_OK) return st;
  const DeviceInfo& di = device_info(dev);
  st = check_device(di);
  if (st != W4_OK) return st;
  MegaLayout L;
  if (!plan_layout(m, di.sm_count, &L))
    return fail(W4_ERR_UNSUPPORTED, "decode model does not fit the step's work split");
  if (scratch == nullptr || scratch_bytes < L.total)
    return fail(W4_ERR_INVALID_ARG, "decode step scratch needs %zu bytes, got %zu", L.total,
                scratch_bytes);
  if (reinterpret_cast<uintptr_t>(scratch) & 255)
    return fail(W4_ERR_ALIGNMENT, "decode step scratch needs 256-byte alignment");

  MegaMaps maps;
  const void* packed[4] = {m.qkv_packed, m.o_packed, m.gu_packed, m.down_packed};
  const void* scales[4] = {m.qkv_scales, m.o_scales, m.gu_scales, m.down_scales};
  for (int i = 0; i < 4; ++i) {
    const MegaGemv& G = L.g[i];
    if (!encode_map(&maps.w[i], CU_TENSOR_MAP_DATA_TYPE_INT32, 4, packed[i], (uint64_t)G.N,
                    (uint64_t)m.layers * (G.K / 8), 32, (uint32_t)(16 * G.bg),
                    CU_TENSOR_MAP_SWIZZLE_128B))
      return fail(W4_ERR_CUDA, "cuTensorMapEncodeTiled failed (decode step weights %d)", i);
    if (!encode_map(&maps.s[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, scales[i], (uint64_t)G.N,
                    (uint64_t)m.layers * G.groups, 32, (uint32_t)G.bg, CU_TENSOR_MAP_SWIZZLE_NONE))
      return fail(W4_ERR_CUDA, "cuTensorMapEncodeTiled failed (decode step scales %d)", i);
  }

  MegaParams p;
  p.layers = m.layers;
  p.hidden = m.hidden;
  p.inter = m.intermediate;
  p.heads = m.heads;
  p.kv_heads = m.kv_heads;
  p.vocab = m.vocab;
  p.max_seq = m.max_seq;
  p.group = m.heads / m.kv_heads;
  p.attn_splits = L.attn_splits;
  p.lm_rows = std::min(8, kSlotBytes / (m.hidden * 2));
  p.eps = m.eps;
  p.scale = 1.0f / sqrtf(128.0f);
  for (int i = 0; i < 4; ++i) p.g[i] = L.g[i];
  p.qkv_bias = static_cast<const uint16_t*>(m.qkv_bias);
  p.in_norm = static_cast<const uint16_t*>(m.in_norm);
  p.post_norm = static_cast<const uint16_t*>(m.post_norm);
  p.final_norm = static_cast<const uint16_t*>(m.final_norm);
  p.embed = static_cast<const uint16_t*>(m.embed);
  p.cos_t = static_cast<const uint16_t*>(m.cos_table);
  p.sin_t = static_cast<const uint16_t*>(m.sin_table);
  p.k_cache = static_cast<uint16_t*>(m.k_cache);
  p.v_cache = static_cast<uint16_t*>(m.v_cache);
  p.prompt = m.prompt;
  p.prompt_len = m.prompt_len;
  p.token = m.token;
  p.pos = m.pos;
  p.logits = static_cast<uint16_t*>(m.logits);
  uint8_t* s = static_cast<uint8_t*>(scratch);
  p.bar = reinterpret_cast<unsigned*>(s);
  p.done = reinterpret_cast<unsigned*>(s + 1024);
  p.best = reinterpret_cast<unsigned long long*>(s + 1152);
  p.h0 = reinterpret_cast<uint16_t*>(s + L.off_h0);
  p.h1 = reinterpret_cast<uint16_t*>(s + L.off_h1);
  for (int i = 0; i < 4; ++i) p.part[i] = reinterpret_cast<float*>(s + L.off_part[i]);
  p.pattn = reinterpret_cast<float*>(s + L.off_attn);
  p.err = di.err_word;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)di.sm_count);
  cfg.blockDim = dim3(kMegaThreads);
  cfg.dynamicSmemBytes = mega_smem_bytes();
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the grid barriers need it
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, decode_step_kernel, maps, p);
  return e == cudaSuccess ? W4_OK : cuda_fail(e, "w4_decode_step launch");
}

}  // namespace w4
