// w4_decode.cu - the non-GEMV kernels of a batch-1 greedy decode step (bf16).
//
// Together with the fused W4A16 GEMV (w4_gemv.cu: RMSNorm / SwiGLU prologues,
// bias / residual epilogues) they replace the HF forward that
// scripts/decode_loop.py:106-124 ran once per token with a `.item()` sync:
//   embed      token selection (prompt or previous argmax) and row gather
//   attention  RoPE on q and k, KV-cache write, GQA attention over 0..pos,
//              split over a thread-block cluster and merged through DSMEM
//   lm_head    final RMSNorm, tied-embedding logits and a deterministic argmax
// Every kernel reads the step state (token, position) from device memory, so a
// whole step is one CUDA-graph replay; with PDL each launch overlaps the
// previous kernel's tail.
#include "w4_internal.h"
#include "w4_ptx.cuh"

#include <cooperative_groups.h>

#include <algorithm>
#include <mutex>

namespace cg = cooperative_groups;

namespace w4 {

namespace {

__device__ __forceinline__ float bf(uint16_t v) { return __uint_as_float((uint32_t)v << 16); }
__device__ __forceinline__ uint16_t to_bf(float v) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}
__device__ __forceinline__ float rbf(float v) { return bf(to_bf(v)); }

cudaLaunchAttribute pdl_attr(int pdl) {
  cudaLaunchAttribute a;
  a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  a.val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  return a;
}

}  // namespace

// ------------------------------------------------------------------ embed

__global__ void __launch_bounds__(256) embed_kernel(const uint16_t* __restrict__ embed, int vocab,
                                                    int hidden, const int64_t* prompt,
                                                    const int64_t* prompt_len, int64_t* token,
                                                    const int64_t* pos, uint16_t* h) {
  grid_dependency_wait();  // token and pos come from the previous step
  const int64_t p = *pos;
  int64_t t = (p < *prompt_len) ? prompt[p] : *token;
  t = t < 0 ? 0 : (t >= vocab ? vocab - 1 : t);  // never read outside the table
  __syncthreads();
  if (blockIdx.x == 0 && threadIdx.x == 0) *token = t;  // the token this step consumes
  const uint4* src = reinterpret_cast<const uint4*>(embed + (size_t)t * hidden);
  uint4* dst = reinterpret_cast<uint4*>(h);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden / 8; i += gridDim.x * blockDim.x)
    dst[i] = __ldg(src + i);
  grid_launch_dependents();
}

int launch_decode_embed(const void* embed, int vocab, int hidden, const int64_t* prompt,
                        const int64_t* prompt_len, int64_t* token, const int64_t* pos, void* h,
                        int pdl, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute at = pdl_attr(pdl);
  cfg.attrs = &at;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, embed_kernel, static_cast<const uint16_t*>(embed),
                                     vocab, hidden, prompt, prompt_len, token, pos,
                                     static_cast<uint16_t*>(h));
  return e == cudaSuccess ? W4_OK : cuda_fail(e, "w4_decode_embed launch");
}

// ------------------------------------------------------------------ attention

// Tensor-core flash decoding. The step's q heads of one KV head form the 16
// rows of an mma.sync m16n8k16 A operand (G <= 16 heads, zero rows above G);
// K rows of 16 positions are its B operand, so the scores of a 16-position
// tile are two 16x8 accumulators per 16 dimensions. Those accumulators are,
// register for register, the A operand of the P.V product (the flash-
// attention layout), so probabilities never leave registers; V rows are read
// with transposing ldmatrix. P enters P.V rounded to bf16, as in the
// reference model's bf16 attention; the softmax sums stay in fp32.
//
// Work split: the positions 0..pos of one KV head are cut into S ranges of at
// most kAttnRows positions (S = ceil(P / kAttnRows), at most kAttnSplits), one
// CTA each; the 8 warps of a CTA take its 16-position tiles round-robin and
// merge in shared memory in warp order. Only when S > 1 do the CTAs of the
// cluster merge over DSMEM in rank order; up to kAttnRows positions one CTA
// per KV head does everything and no cluster barrier is run. The cached rows
// below pos were written by earlier steps, so they are copied into shared
// memory before the grid-dependency wait.
constexpr int kAttnSplits = 8;   // CTAs (cluster) per KV head
constexpr int kHeadDim = 128;
constexpr int kAttnWarps = 8;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kAttnRows = 256;       // positions per shared-memory pass of one CTA
constexpr int kRowBytes = kHeadDim * 2;  // one K or V row, 16 chunks of 16 bytes
constexpr int kObPitch = kHeadDim + 4;   // floats per row of the warp-merge buffer
constexpr int kAttnTilesPerWarp = 1;     // 16-position tiles per warp before another joins

struct AttnParams {
  const uint16_t* qkv;  // [heads*hd | kv*hd | kv*hd]
  const uint16_t* cos_t;
  const uint16_t* sin_t;  // [max_seq, hd]
  const int64_t* pos;
  uint16_t* k_cache;
  uint16_t* v_cache;  // [kv, max_seq, hd]
  uint16_t* out;      // [heads*hd]
  int heads, kv_heads, max_seq, group;  // group = heads / kv_heads
  float scale_log2;                     // log2(e) / sqrt(hd)
};

// RoPE (rotate-half) of dimension d of one head, in the reference model's
// bf16 arithmetic: round(x*cos) + round(rot(x)*sin), rounded.
__device__ __forceinline__ float rope_dim(const uint16_t* head, int d, float c, float s) {
  const float x = bf(head[d]);
  const float partner = bf(head[d ^ 64]);
  const float rot = (d < 64) ? -partner : partner;
  return rbf(rbf(x * c) + rbf(rot * s));
}

// Byte offset of 16-byte chunk `chunk` of row `row` in a buffer of 256-byte
// rows: the chunk index is XOR-ed with the row's low 3 bits, so the 8 rows an
// ldmatrix reads at one chunk fall on 8 different bank groups.
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return (uint32_t)(row * kRowBytes + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void cp_async16_attn(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return (uint32_t)to_bf(lo) | ((uint32_t)to_bf(hi) << 16);
}

// Shared memory (attn_smem_bytes):
//   kbuf, vbuf  bf16 [kAttnRows][128], swizzled   K and V rows of the pass
//               (after the last pass: the warp-merge buffer ob, f32
//               [kAttnWarps][G][kObPitch], aliases them)
//   qbuf        bf16 [16][128], swizzled          q after RoPE, rows >= G zero
//   raw         bf16 [G + 2][128]                 this token's q heads, k, v
//   kvnew       bf16 [2][128]                     this token's k (after RoPE) and v
//   cs          f32 [2][128]                      cos and sin of the position
//   wm, wl      f32 [kAttnWarps][16]              per-warp row max and sum
//   rm, rl      f32 [16]                          the CTA's row max and sum
//   cpart       f32 [G][128]                      the CTA's unnormalised output
static size_t attn_smem_bytes(int G) {
  const size_t kv = 2 * (size_t)kAttnRows * kRowBytes;
  const size_t ob = (size_t)kAttnWarps * G * kObPitch * 4;
  return std::max(kv, ob) + 16 * kRowBytes + (size_t)(G + 2) * kRowBytes + 2 * kRowBytes +
         2 * kHeadDim * 4 + (2 * kAttnWarps * 16 + 2 * 16) * 4 + (size_t)G * kHeadDim * 4 + 128;
}

__global__ void __launch_bounds__(kAttnThreads, 1) attention_kernel(const AttnParams p) {
  extern __shared__ __align__(128) unsigned char smem_attn[];
  const int G = p.group;
  const int kvh = blockIdx.x;
  const int rank = blockIdx.y;  // the cluster spans the splits of one KV head
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;

  uint8_t* kbuf = smem_attn;
  uint8_t* vbuf = kbuf + (size_t)kAttnRows * kRowBytes;
  float* ob = reinterpret_cast<float*>(smem_attn);  // after the last pass
  uint8_t* qbuf = smem_attn + std::max((size_t)2 * kAttnRows * kRowBytes,
                                       (size_t)kAttnWarps * G * kObPitch * 4);
  uint16_t* raw = reinterpret_cast<uint16_t*>(qbuf + 16 * kRowBytes);
  uint16_t* kvnew = raw + (G + 2) * kHeadDim;
  float* cs = reinterpret_cast<float*>(kvnew + 2 * kHeadDim);
  float* wm = cs + 2 * kHeadDim;
  float* wl = wm + kAttnWarps * 16;
  float* rm = wl + kAttnWarps * 16;
  float* rl = rm + 16;
  float* cpart = rl + 16;
  const uint32_t k_s = smem_u32(kbuf), v_s = smem_u32(vbuf), q_s = smem_u32(qbuf);

  // The position and the cached rows below it were written by earlier steps.
  const int64_t raw_pos = *p.pos;
  // a position outside the cache is clamped (wrong output, never a wild store)
  const int pos = raw_pos < 0 ? 0 : (raw_pos >= p.max_seq ? p.max_seq - 1 : (int)raw_pos);
  const int P = pos + 1;
  const int S = min(kAttnSplits, (P + kAttnRows - 1) / kAttnRows);
  int chunk = (P + S - 1) / S;
  chunk = (chunk + 15) & ~15;
  const int j0 = min(P, rank * chunk), j1 = min(P, j0 + chunk);
  if (rank >= S && S == 1) return;  // no merge: the other CTAs have nothing to do
  const uint16_t* kc = p.k_cache + (size_t)kvh * p.max_seq * kHeadDim;
  const uint16_t* vc = p.v_cache + (size_t)kvh * p.max_seq * kHeadDim;

  // First pass of cached rows [j0, min(j1, pos)), 16-byte asynchronous copies.
  {
    const int r1 = min(min(j1, j0 + kAttnRows), pos);
    for (int i = tid; i < (r1 - j0) * 16; i += kAttnThreads) {
      const int r = i >> 4, c = i & 15;
      cp_async16_attn(k_s + swz(r, c), kc + (size_t)(j0 + r) * kHeadDim + 8 * c);
      cp_async16_attn(v_s + swz(r, c), vc + (size_t)(j0 + r) * kHeadDim + 8 * c);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  {  // cos (threads 0..127) and sin (128..255) of the position
    const uint16_t* tab = tid < kHeadDim ? p.cos_t : p.sin_t;
    cs[tid] = bf(tab[(size_t)pos * kHeadDim + (tid & (kHeadDim - 1))]);
  }
  grid_launch_dependents();  // the o projection may start streaming its weights

  grid_dependency_wait();  // q/k/v come from the previous kernel
  {
    const uint4* q = reinterpret_cast<const uint4*>(p.qkv + (size_t)kvh * G * kHeadDim);
    const uint4* k = reinterpret_cast<const uint4*>(p.qkv + (size_t)(p.heads + kvh) * kHeadDim);
    const uint4* v =
        reinterpret_cast<const uint4*>(p.qkv + (size_t)(p.heads + p.kv_heads + kvh) * kHeadDim);
    uint4* dst = reinterpret_cast<uint4*>(raw);
    for (int i = tid; i < (G + 2) * 16; i += kAttnThreads) {
      const int h = i >> 4, cc = i & 15;
      dst[i] = __ldcg((h < G ? q + h * 16 : (h == G ? k : v)) + cc);
    }
  }
  __syncthreads();
  // RoPE over every thread: the q heads into the swizzled A operand, k into
  // kvnew[0], v copied to kvnew[1]; the CTA that owns the new position also
  // stores its k and v in the cache. Rows G..15 of the A operand are zero.
  const bool owner = pos >= j0 && pos < j1;
  for (int e = tid; e < (G + 2) * kHeadDim; e += kAttnThreads) {
    const int h = e >> 7, d = e & (kHeadDim - 1);
    if (h < G) {
      *reinterpret_cast<uint16_t*>(qbuf + swz(h, d >> 3) + 2 * (d & 7)) =
          to_bf(rope_dim(raw + h * kHeadDim, d, cs[d], cs[kHeadDim + d]));
    } else {
      const uint16_t val = h == G ? to_bf(rope_dim(raw + h * kHeadDim, d, cs[d], cs[kHeadDim + d]))
                                  : raw[h * kHeadDim + d];
      kvnew[(h - G) * kHeadDim + d] = val;
      if (owner) {  // this CTA owns the new position: store it
        const size_t at = ((size_t)kvh * p.max_seq + pos) * kHeadDim + d;
        (h == G ? p.k_cache : p.v_cache)[at] = val;
      }
    }
  }
  for (int i = tid; i < (16 - G) * 16; i += kAttnThreads)
    *reinterpret_cast<uint4*>(qbuf + swz(G + (i >> 4), i & 15)) = make_uint4(0u, 0u, 0u, 0u);
  __syncthreads();

  // q fragments (A operand), one set of 4 registers per 16 dimensions
  uint32_t qa[8][4];
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // rows g and g + 8

  // Warps that take tiles: with one pass, about kAttnTilesPerWarp tiles each,
  // in contiguous runs (a short context needs fewer warps, and with one warp
  // the cross-warp merge is skipped); with several passes all warps,
  // round-robin.
  const bool one_pass = j1 - j0 <= kAttnRows;
  const int nt_first = (min(j1 - j0, kAttnRows) + 15) >> 4;
  const int W = one_pass ? max(1, min(kAttnWarps, (nt_first + kAttnTilesPerWarp - 1) /
                                                      kAttnTilesPerWarp))
                         : kAttnWarps;
  for (int b0 = j0; b0 < j1; b0 += kAttnRows) {  // passes over this CTA's range
    const int b1 = min(j1, b0 + kAttnRows);
    const int n = b1 - b0;
    if (b0 != j0) {  // later passes (more than kAttnRows positions per CTA)
      __syncthreads();  // the previous pass is consumed
      const int r1 = min(b1, pos);
      for (int i = tid; i < (r1 - b0) * 16; i += kAttnThreads) {
        const int r = i >> 4, c = i & 15;
        cp_async16_attn(k_s + swz(r, c), kc + (size_t)(b0 + r) * kHeadDim + 8 * c);
        cp_async16_attn(v_s + swz(r, c), vc + (size_t)(b0 + r) * kHeadDim + 8 * c);
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (tid < 32 && pos >= b0 && pos < b1) {  // the new position's row, 16-byte chunks
      const int r = pos - b0, c = tid & 15;
      const uint4 v = reinterpret_cast<const uint4*>(kvnew + (tid >> 4) * kHeadDim)[c];
      *reinterpret_cast<uint4*>((tid < 16 ? kbuf : vbuf) + swz(r, c)) = v;
    }
    // rows past the range up to the tile boundary: zeros (a masked probability
    // times stale shared memory could otherwise be 0 * NaN)
    for (int i = tid; i < (((n + 15) & ~15) - n) * 16; i += kAttnThreads) {
      const int r = n + (i >> 4), c = i & 15;
      *reinterpret_cast<uint4*>(kbuf + swz(r, c)) = make_uint4(0u, 0u, 0u, 0u);
      *reinterpret_cast<uint4*>(vbuf + swz(r, c)) = make_uint4(0u, 0u, 0u, 0u);
    }
    __syncthreads();
    if (b0 == j0) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        ldsm_x4(q_s + swz((lane & 7) + ((lane >> 3) & 1) * 8, 2 * ks + (lane >> 4)), qa[ks]);
    }
    const int n_tiles = (n + 15) >> 4;
    const int tpw = (n_tiles + W - 1) / W;
    const int t_begin = one_pass ? warp * tpw : warp;
    const int t_end = one_pass ? min(n_tiles, t_begin + tpw) : n_tiles;
    const int t_step = one_pass ? 1 : kAttnWarps;
    for (int tile = t_begin; tile < t_end; tile += t_step) {
      const int r0 = tile * 16;
      // scores S^T[head][position] of 16 positions: two 16x8 accumulators
      float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t kb[4];
        ldsm_x4(k_s + swz(r0 + (lane & 7) + ((lane >> 4) & 1) * 8, 2 * ks + ((lane >> 3) & 1)),
                kb);
        mma_16816<true>(s[0], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], kb[0], kb[1]);
        mma_16816<true>(s[1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], kb[2], kb[3]);
      }
      // scale to log2 units, mask positions past the range
#pragma unroll
      for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int col = r0 + 8 * a + 2 * t + (i & 1);
          s[a][i] = col < n ? s[a][i] * p.scale_log2 : -INFINITY;
        }
      float t0 = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
      float t1 = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
#pragma unroll
      for (int off = 1; off <= 2; off <<= 1) {
        t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, off));
        t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, off));
      }
      const float n0 = fmaxf(m0, t0), n1 = fmaxf(m1, t1);  // finite: a tile holds >= 1 position
      const float al0 = exp2f(m0 - n0), al1 = exp2f(m1 - n1);  // 0 while m is -inf
      m0 = n0;
      m1 = n1;
      float pr[2][4];
#pragma unroll
      for (int a = 0; a < 2; ++a) {
        pr[a][0] = exp2f(s[a][0] - n0);
        pr[a][1] = exp2f(s[a][1] - n0);
        pr[a][2] = exp2f(s[a][2] - n1);
        pr[a][3] = exp2f(s[a][3] - n1);
      }
      l0 = l0 * al0 + ((pr[0][0] + pr[0][1]) + (pr[1][0] + pr[1][1]));
      l1 = l1 * al1 + ((pr[0][2] + pr[0][3]) + (pr[1][2] + pr[1][3]));
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        o[j][0] *= al0;
        o[j][1] *= al0;
        o[j][2] *= al1;
        o[j][3] *= al1;
      }
      // P as the A operand (rows = heads, k = the 16 positions), rounded to
      // bf16 as the reference model's attention does before P.V; the row sums
      // l stay in fp32
      uint32_t ph[4];
      const float* src[4] = {&pr[0][0], &pr[0][2], &pr[1][0], &pr[1][2]};
#pragma unroll
      for (int r = 0; r < 4; ++r) ph[r] = pack_bf16x2(src[r][0], src[r][1]);
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {  // 16 dimensions per transposing ldmatrix
        uint32_t vb[4];
        ldsm_x4_t(v_s + swz(r0 + (lane & 7) + ((lane >> 3) & 1) * 8, 2 * jj + (lane >> 4)), vb);
        mma_16816<true>(o[2 * jj], ph[0], ph[1], ph[2], ph[3], vb[0], vb[1]);
        mma_16816<true>(o[2 * jj + 1], ph[0], ph[1], ph[2], ph[3], vb[2], vb[3]);
      }
    }
  }

  // ---- merge the warps (fixed warp order)
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  if (W == 1) {  // warp 0 holds every position of this CTA: no cross-warp merge
    if (S == 1) {
      if (warp == 0) {
        // rows < G saw at least one position, so l >= 1
        const float i0 = 1.0f / l0, i1 = 1.0f / l1;
        uint16_t* out = p.out + (size_t)kvh * G * kHeadDim;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (g < G)
            *reinterpret_cast<uint32_t*>(out + g * kHeadDim + 8 * j + 2 * t) =
                pack_bf16x2(o[j][0] * i0, o[j][1] * i0);
          if (g + 8 < G)
            *reinterpret_cast<uint32_t*>(out + (g + 8) * kHeadDim + 8 * j + 2 * t) =
                pack_bf16x2(o[j][2] * i1, o[j][3] * i1);
        }
      }
      return;
    }
    if (warp == 0) {  // this CTA's partial for the cluster merge
      if (t == 0) {
        rm[g] = m0;
        rm[g + 8] = m1;
        rl[g] = l0;
        rl[g + 8] = l1;
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if (g < G)
          *reinterpret_cast<float2*>(cpart + g * kHeadDim + 8 * j + 2 * t) =
              make_float2(o[j][0], o[j][1]);
        if (g + 8 < G)
          *reinterpret_cast<float2*>(cpart + (g + 8) * kHeadDim + 8 * j + 2 * t) =
              make_float2(o[j][2], o[j][3]);
      }
    }
  } else {
    if (t == 0) {
      wm[warp * 16 + g] = m0;
      wm[warp * 16 + g + 8] = m1;
      wl[warp * 16 + g] = l0;
      wl[warp * 16 + g + 8] = l1;
    }
    __syncthreads();  // every warp is past its last tile: kbuf/vbuf become ob
    float M0 = -INFINITY, M1 = -INFINITY;
    for (int w = 0; w < kAttnWarps; ++w) {
      M0 = fmaxf(M0, wm[w * 16 + g]);
      M1 = fmaxf(M1, wm[w * 16 + g + 8]);
    }
    if (tid < 16) {
      float M = -INFINITY, L = 0.f;
      for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, wm[w * 16 + tid]);
      for (int w = 0; w < kAttnWarps; ++w) {
        const float mw = wm[w * 16 + tid];
        if (mw != -INFINITY) L = fmaf(wl[w * 16 + tid], exp2f(mw - M), L);
      }
      rm[tid] = M;
      rl[tid] = L;
    }
    const float f0 = (m0 == -INFINITY) ? 0.f : exp2f(m0 - M0);
    const float f1 = (m1 == -INFINITY) ? 0.f : exp2f(m1 - M1);
    if (warp < W) {
  #pragma unroll
      for (int j = 0; j < 16; ++j) {
        if (g < G)
          *reinterpret_cast<float2*>(ob + ((size_t)warp * G + g) * kObPitch + 8 * j + 2 * t) =
              make_float2(o[j][0] * f0, o[j][1] * f0);
        if (g + 8 < G)
          *reinterpret_cast<float2*>(ob + ((size_t)warp * G + g + 8) * kObPitch + 8 * j + 2 * t) =
              make_float2(o[j][2] * f1, o[j][3] * f1);
      }
    }
    __syncthreads();
    for (int e = tid; e < G * kHeadDim; e += kAttnThreads) {
      const int h = e >> 7, d = e & (kHeadDim - 1);
      float acc = 0.f;
      for (int w = 0; w < W; ++w) acc += ob[((size_t)w * G + h) * kObPitch + d];
      if (S == 1)
        p.out[(size_t)(kvh * G + h) * kHeadDim + d] = to_bf(acc / rl[h]);
      else
        cpart[e] = acc;
    }
    if (S == 1) return;
  }

  // ---- merge the CTAs of this KV head over DSMEM (rank order); an idle CTA
  // (rank >= S) contributes m = -inf, l = 0
  if (rank >= S && tid < 16) {
    rm[tid] = -INFINITY;
    rl[tid] = 0.f;
  }
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  for (int e = rank * kAttnThreads + tid; e < G * kHeadDim; e += kAttnThreads * kAttnSplits) {
    const int h = e >> 7;
    float M = -INFINITY;
    for (int r = 0; r < S; ++r) M = fmaxf(M, cluster.map_shared_rank(rm, r)[h]);
    float L = 0.f, O = 0.f;
    for (int r = 0; r < S; ++r) {
      const float mr = cluster.map_shared_rank(rm, r)[h];
      const float w = (mr == -INFINITY) ? 0.f : exp2f(mr - M);
      L = fmaf(w, cluster.map_shared_rank(rl, r)[h], L);
      O = fmaf(w, cluster.map_shared_rank(cpart, r)[e], O);
    }
    p.out[(size_t)(kvh * G + h) * kHeadDim + (e & (kHeadDim - 1))] = to_bf(O / L);
  }
  cluster.sync();  // keep this CTA's shared memory alive for the readers
}

int launch_decode_attention(const void* qkv, const void* cos_t, const void* sin_t,
                            const int64_t* pos, void* k_cache, void* v_cache, void* out, int heads,
                            int kv_heads, int max_seq, int pdl, cudaStream_t stream) {
  AttnParams p;
  p.qkv = static_cast<const uint16_t*>(qkv);
  p.cos_t = static_cast<const uint16_t*>(cos_t);
  p.sin_t = static_cast<const uint16_t*>(sin_t);
  p.pos = pos;
  p.k_cache = static_cast<uint16_t*>(k_cache);
  p.v_cache = static_cast<uint16_t*>(v_cache);
  p.out = static_cast<uint16_t*>(out);
  p.heads = heads;
  p.kv_heads = kv_heads;
  p.max_seq = max_seq;
  p.group = heads / kv_heads;
  p.scale_log2 = 1.4426950408889634f / sqrtf((float)kHeadDim);
  const size_t smem = attn_smem_bytes(p.group);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)kv_heads, kAttnSplits, 1);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 1;
  at[0].val.clusterDim.y = kAttnSplits;
  at[0].val.clusterDim.z = 1;
  at[1] = pdl_attr(pdl);
  cfg.attrs = at;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, attention_kernel, p);
  return e == cudaSuccess ? W4_OK : cuda_fail(e, "w4_decode_attention launch");
}

// ------------------------------------------------------------------ lm_head + argmax

// One persistent CTA per SM streams a contiguous range of embedding rows
// (the tied lm_head) through a ring of shared-memory stages filled by 1-D
// bulk copies; 16 consumer warps turn each stage's rows into logits (one row
// each per 16-row stage: 73.6 us per 467 MB chained, against 75.9 with 8
// warps taking two rows each).
constexpr int kLmConsumerWarps = 16;
constexpr int kLmThreads = (kLmConsumerWarps + 1) * 32;
constexpr int kLmRowsPerStage = 16;
// ring depth: 4 stages of 16 rows (192 KB at hidden 1536), 3 for hidden 2048
__host__ __device__ constexpr int lm_stages(int hidden) { return hidden <= 1536 ? 4 : 3; }

struct LmHeadWorkspace {
  unsigned long long best;  // (ordered bf16 logit << 32) | (0xffffffff - index)
  unsigned int done;        // CTAs finished this step
  unsigned int pad[13];
};

size_t lm_head_workspace_bytes() { return sizeof(LmHeadWorkspace); }

// Monotonic map of a float's bits to unsigned (larger float -> larger key).
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

static size_t lm_smem_bytes(int hidden) {
  return 128 + (size_t)lm_stages(hidden) * kLmRowsPerStage * hidden * 2 + (size_t)hidden * 4 +
         2 * lm_stages(hidden) * sizeof(uint64_t);
}

template <int CH>  // CH = hidden / 256: 16-byte chunks per lane per row
__global__ void __launch_bounds__(kLmThreads, 1) lm_head_kernel(
    const uint16_t* __restrict__ h, const uint16_t* __restrict__ norm_w, float eps,
    const uint16_t* __restrict__ embed, int vocab, uint16_t* __restrict__ logits,
    int64_t* token, int64_t* pos, LmHeadWorkspace* ws, int* err) {
  constexpr int H = CH * 256;
  constexpr uint32_t kRowBytes = H * 2;
  constexpr int kLmStages = lm_stages(H);
  extern __shared__ __align__(128) unsigned char smem_lm[];
  uint8_t* stage_s = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_lm) + 127) & ~static_cast<uintptr_t>(127));
  float* x_s = reinterpret_cast<float*>(stage_s + kLmStages * kLmRowsPerStage * kRowBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(x_s + H);
  uint64_t* empty = full + kLmStages;
  __shared__ float red[kLmConsumerWarps];
  __shared__ unsigned long long best_s[kLmConsumerWarps];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // this CTA's rows
  const int per = (vocab + gridDim.x - 1) / gridDim.x;
  const int r0 = min(vocab, blockIdx.x * per), r1 = min(vocab, r0 + per);
  const int n_stages = (r1 - r0 + kLmRowsPerStage - 1) / kLmRowsPerStage;

  if (tid == 0) {
    for (int s = 0; s < kLmStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kLmConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  unsigned long long best = 0;
  if (warp == kLmConsumerWarps) {
    // producer: the embedding is constant, so it streams before the grid
    // dependency is resolved
    grid_launch_dependents();
    if (lane == 0) {
      int slot = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int j = 0; j < n_stages; ++j) {
        if (j >= kLmStages && !mbar_wait(&empty[slot], phase ^ 1u)) {
          if (err) atomicCAS(err, 0, kErrEmptyWait);
          break;
        }
        const int rs = r0 + j * kLmRowsPerStage;
        const uint32_t bytes = (uint32_t)min(kLmRowsPerStage, r1 - rs) * kRowBytes;
        mbar_arrive_expect_tx(&full[slot], bytes);
        bulk_load(stage_s + (size_t)slot * kLmRowsPerStage * kRowBytes,
                  embed + (size_t)rs * H, bytes, &full[slot]);
        ++issued;
        if (++slot == kLmStages) {
          slot = 0;
          phase ^= 1u;
        }
      }
      for (int j = max(0, issued - kLmStages); j < issued; ++j)  // no copy left in flight
        if (!mbar_wait(&full[j % kLmStages], (j / kLmStages) & 1) && err)
          atomicCAS(err, 0, kErrDrainWait);
    }
  } else {
    grid_dependency_wait();  // h comes from the previous kernel
    // final RMSNorm (fp32 normalisation, cast to bf16, times the bf16 weight)
    float ss = 0.f;
    for (int i = tid; i < H; i += kLmConsumerWarps * 32) {
      const float v = bf(h[i]);
      ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) red[warp] = ss;
    asm volatile("bar.sync 1, %0;" ::"r"(kLmConsumerWarps * 32) : "memory");
    float tot = 0.f;
    for (int w = 0; w < kLmConsumerWarps; ++w) tot += red[w];
    const float inv = rsqrtf(tot / (float)H + eps);
    for (int i = tid; i < H; i += kLmConsumerWarps * 32)
      x_s[i] = rbf(rbf(bf(h[i]) * inv) * bf(norm_w[i]));
    asm volatile("bar.sync 1, %0;" ::"r"(kLmConsumerWarps * 32) : "memory");
    grid_launch_dependents();  // every thread signals (the producer warp below)

    // lane l owns elements 8*(32*c + l) .. +7 of every row
    float xr[CH][8];
#pragma unroll
    for (int c = 0; c < CH; ++c)
#pragma unroll
      for (int i = 0; i < 8; ++i) xr[c][i] = x_s[8 * (32 * c + lane) + i];

    int slot = 0;
    uint32_t phase = 0;
    for (int j = 0; j < n_stages; ++j) {
      if (!mbar_wait(&full[slot], phase)) {
        if (err) atomicCAS(err, 0, kErrFullWait);
        break;
      }
      const int rs = r0 + j * kLmRowsPerStage;
      const int nrows = min(kLmRowsPerStage, r1 - rs);
      const uint8_t* st = stage_s + (size_t)slot * kLmRowsPerStage * kRowBytes;
      // warp w takes rows w and w + 8 of the stage (two dot products in flight)
      for (int rl = warp; rl < nrows; rl += 2 * kLmConsumerWarps) {
        const int rl2 = rl + kLmConsumerWarps;
        const bool two = rl2 < nrows;
        const uint4* ra = reinterpret_cast<const uint4*>(st + (size_t)rl * kRowBytes);
        const uint4* rb = reinterpret_cast<const uint4*>(st + (size_t)(two ? rl2 : rl) * kRowBytes);
        float da = 0.f, db = 0.f;
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          const uint4 a = ra[32 * c + lane], b = rb[32 * c + lane];
          const uint32_t* av = reinterpret_cast<const uint32_t*>(&a);
          const uint32_t* bv = reinterpret_cast<const uint32_t*>(&b);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            da = fmaf(bf(av[i] & 0xffffu), xr[c][2 * i], da);
            da = fmaf(bf(av[i] >> 16), xr[c][2 * i + 1], da);
            db = fmaf(bf(bv[i] & 0xffffu), xr[c][2 * i], db);
            db = fmaf(bf(bv[i] >> 16), xr[c][2 * i + 1], db);
          }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
          da += __shfl_xor_sync(0xffffffffu, da, off);
          db += __shfl_xor_sync(0xffffffffu, db, off);
        }
        if (lane == 0) {
          // argmax over the bf16 logits, first index among equals
          const int ia = rs + rl, ib = rs + rl2;
          const uint16_t la = to_bf(da);
          if (logits) logits[ia] = la;
          const unsigned long long ka =
              ((unsigned long long)order_key(bf(la)) << 32) | (0xffffffffu - (uint32_t)ia);
          best = ka > best ? ka : best;
          if (two) {
            const uint16_t lb = to_bf(db);
            if (logits) logits[ib] = lb;
            const unsigned long long kb =
                ((unsigned long long)order_key(bf(lb)) << 32) | (0xffffffffu - (uint32_t)ib);
            best = kb > best ? kb : best;
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      if (++slot == kLmStages) {
        slot = 0;
        phase ^= 1u;
      }
    }
    if (lane == 0) best_s[warp] = best;
  }
  __syncthreads();
  if (tid == 0) {
    unsigned long long b = 0;
    for (int w = 0; w < kLmConsumerWarps; ++w) b = best_s[w] > b ? best_s[w] : b;
    atomicMax(&ws->best, b);
    __threadfence();
    const unsigned int ticket = atomicAdd(&ws->done, 1u);
    if (ticket == gridDim.x - 1) {  // last CTA: every other CTA's max is visible
      __threadfence();
      const unsigned long long fin = atomicAdd(&ws->best, 0ull);
      *token = (int64_t)(0xffffffffu - (uint32_t)(fin & 0xffffffffu));
      *pos = *pos + 1;
      ws->best = 0;  // leave the workspace zeroed for the next step
      ws->done = 0;
      __threadfence();
    }
  }
}

int launch_lm_head_argmax(const void* h, const void* norm_w, float eps, const void* embed,
                          int vocab, int hidden, void* logits, int64_t* token, int64_t* pos,
                          void* workspace, int pdl, cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  const DeviceInfo& di = device_info(dev);
  const int sms = di.sm_count > 0 ? di.sm_count : 148;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)sms);
  cfg.blockDim = dim3(kLmThreads);
  cfg.dynamicSmemBytes = lm_smem_bytes(hidden);
  cfg.stream = stream;
  if (cfg.dynamicSmemBytes > (size_t)di.max_smem_optin)
    return fail(W4_ERR_UNSUPPORTED, "w4_lm_head_argmax: hidden %d needs %zu B of shared memory",
                hidden, cfg.dynamicSmemBytes);
  cudaLaunchAttribute at = pdl_attr(pdl);
  cfg.attrs = &at;
  cfg.numAttrs = 1;
  const uint16_t* hh = static_cast<const uint16_t*>(h);
  const uint16_t* nw = static_cast<const uint16_t*>(norm_w);
  const uint16_t* em = static_cast<const uint16_t*>(embed);
  uint16_t* lg = static_cast<uint16_t*>(logits);
  LmHeadWorkspace* ws = static_cast<LmHeadWorkspace*>(workspace);
  int* err = di.err_word;
  cudaError_t e;
  switch (hidden / 256) {
    case 1: e = cudaLaunchKernelEx(&cfg, lm_head_kernel<1>, hh, nw, eps, em, vocab, lg, token, pos, ws, err); break;
    case 2: e = cudaLaunchKernelEx(&cfg, lm_head_kernel<2>, hh, nw, eps, em, vocab, lg, token, pos, ws, err); break;
    case 4: e = cudaLaunchKernelEx(&cfg, lm_head_kernel<4>, hh, nw, eps, em, vocab, lg, token, pos, ws, err); break;
    case 6: e = cudaLaunchKernelEx(&cfg, lm_head_kernel<6>, hh, nw, eps, em, vocab, lg, token, pos, ws, err); break;
    case 8: e = cudaLaunchKernelEx(&cfg, lm_head_kernel<8>, hh, nw, eps, em, vocab, lg, token, pos, ws, err); break;
    default:
      return fail(W4_ERR_UNSUPPORTED,
                  "w4_lm_head_argmax: hidden %d not in {256, 512, 1024, 1536, 2048}", hidden);
  }
  return e == cudaSuccess ? W4_OK : cuda_fail(e, "w4_lm_head_argmax launch");
}

// ------------------------------------------------------------------ allocation-free lm_head
//
// Some hosts cannot hand this library device memory: a C or C++ decode loop
// embedded in a process whose device memory is owned by someone else's pool,
// or a plugin that is not allowed to call an allocator once serving has
// started. For them the argmax state of the lm_head kernel lives in a fixed
// array that the module itself provides. Every call on a device shares that
// one array, so calls that overlap on the GPU race with each other.
constexpr size_t kStaticScratchBytes = W4B200_STATIC_SCRATCH_BYTES;
static_assert(sizeof(LmHeadWorkspace) <= kStaticScratchBytes,
              "the lm_head argmax state must fit the static scratch");
static __device__ __align__(256) unsigned char g_lm_head_scratch[kStaticScratchBytes];

namespace {
std::mutex g_static_scratch_mutex;
void* g_static_scratch[64] = {};  // device address of g_lm_head_scratch, per device
}  // namespace

int lm_head_argmax_static(const void* h, const void* norm_w, float eps, const void* embed,
                          int vocab, int hidden, void* logits, int64_t* token, int64_t* pos,
                          int pdl, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(W4_ERR_UNSUPPORTED, "device %d", dev);
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_static_scratch_mutex);
    if (!g_static_scratch[dev]) {
      // In host code g_lm_head_scratch only names the array; the kernel needs
      // its address on this device.
      e = cudaGetSymbolAddress(&scratch, g_lm_head_scratch);
      if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(lm_head scratch)");
      // The array is zero when the module loads and every finished call
      // leaves it zero; clearing it here also recovers from a call that was
      // cut short.
      e = cudaMemsetAsync(scratch, 0, sizeof(LmHeadWorkspace), stream);
      if (e != cudaSuccess) return cuda_fail(e, "clearing the lm_head scratch");
      g_static_scratch[dev] = scratch;
    }
    scratch = g_static_scratch[dev];
  }
  return launch_lm_head_argmax(h, norm_w, eps, embed, vocab, hidden, logits, token, pos,
                               scratch, pdl, stream);
}

int decode_init_device(const DeviceInfo& di) {
  const int lm_smem = (int)std::min<size_t>(lm_smem_bytes(2048), (size_t)di.max_smem_optin);
  const void* lm_kernels[] = {(const void*)lm_head_kernel<1>, (const void*)lm_head_kernel<2>,
                              (const void*)lm_head_kernel<4>, (const void*)lm_head_kernel<6>,
                              (const void*)lm_head_kernel<8>};
  for (const void* k : lm_kernels) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, lm_smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(lm_head smem)");
  }
  // the same carveout as the GEMV kernels, so PDL-chained grids share SMs
  const void* all[] = {(const void*)lm_head_kernel<1>, (const void*)lm_head_kernel<2>,
                       (const void*)lm_head_kernel<4>, (const void*)lm_head_kernel<6>,
                       (const void*)lm_head_kernel<8>, (const void*)attention_kernel,
                       (const void*)embed_kernel};
  for (const void* k : all) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout,
                                         cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(carveout)");
  }
  const size_t smem = attn_smem_bytes(16);
  cudaError_t e = cudaFuncSetAttribute(attention_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)std::min<size_t>(smem, (size_t)di.max_smem_optin));
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(attention smem)");
  return W4_OK;
}

}  // namespace w4
