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

// Splits of the position range per KV head, one thread-block cluster.
constexpr int kAttnSplits = 8;
constexpr int kHeadDim = 128;
constexpr int kAttnThreads = 128;  // thread i owns dimension i in the RoPE phase

struct AttnParams {
  const uint16_t* qkv;  // [heads*hd | kv*hd | kv*hd]
  const uint16_t* cos_t;
  const uint16_t* sin_t;  // [max_seq, hd]
  const int64_t* pos;
  uint16_t* k_cache;
  uint16_t* v_cache;  // [kv, max_seq, hd]
  uint16_t* out;      // [heads*hd]
  int heads, kv_heads, max_seq, group;  // group = heads / kv_heads
  float scale;
};

// RoPE (rotate-half) of dimension d of one head, in the reference model's
// bf16 arithmetic: round(x*cos) + round(rot(x)*sin), rounded.
__device__ __forceinline__ float rope_dim(const uint16_t* head, int d, float c, float s) {
  const float x = bf(head[d]);
  const float partner = bf(head[d ^ 64]);
  const float rot = (d < 64) ? -partner : partner;
  return rbf(rbf(x * c) + rbf(rot * s));
}

// Positions per shared-memory tile of the split's K/V range.
constexpr int kAttnTile = 64;
constexpr int kKPitch = kHeadDim + 2;  // bf16 per K row: +1 word, conflict-free column reads
constexpr int kQPitch = kHeadDim + 4;  // floats per q row: rows land on different banks

// Shared memory layout (attn_smem_bytes gives its size):
//   raw   bf16 [(G + 2) * 128]           this token's q (G heads), k, v
//   q_s   f32  [G][kQPitch]              q after RoPE
//   kn_s  f32  [128], vn_s f32 [128]     this token's k (after RoPE) and v
//   kt_s  bf16 [kAttnTile][kKPitch]      K rows of the current tile
//   vt_s  bf16 [kAttnTile][128]          V rows of the current tile
//   sc_s  f32  [kAttnTile][G]            scores, then probabilities, of the tile
//   hm_s, hl_s, ha_s  f32 [G]            running max, sum and rescale factor
//   pm_s, pl_s f32 [G], po_s f32 [G][128]  this split's partial result
struct AttnSmem {
  uint16_t* raw;
  float* q_s;
  float* kn_s;
  float* vn_s;
  uint16_t* kt_s;
  uint16_t* vt_s;
  float* sc_s;
  float* hm_s;
  float* hl_s;
  float* ha_s;
  float* pm_s;
  float* pl_s;
  float* po_s;
};

__host__ __device__ inline size_t attn_raw_bytes(int G) {
  return ((size_t)(G + 2) * kHeadDim * 2 + 15) / 16 * 16;
}

__device__ __forceinline__ AttnSmem attn_layout(unsigned char* base, int G) {
  AttnSmem m;
  m.raw = reinterpret_cast<uint16_t*>(base);
  m.q_s = reinterpret_cast<float*>(base + attn_raw_bytes(G));
  m.kn_s = m.q_s + G * kQPitch;
  m.vn_s = m.kn_s + kHeadDim;
  m.kt_s = reinterpret_cast<uint16_t*>(m.vn_s + kHeadDim);
  m.vt_s = m.kt_s + kAttnTile * kKPitch;
  m.sc_s = reinterpret_cast<float*>(m.vt_s + kAttnTile * kHeadDim);
  m.hm_s = m.sc_s + kAttnTile * G;
  m.hl_s = m.hm_s + G;
  m.ha_s = m.hl_s + G;
  m.pm_s = m.ha_s + G;
  m.pl_s = m.pm_s + G;
  m.po_s = m.pl_s + G;
  return m;
}

static size_t attn_smem_bytes(int G) {
  const size_t f32 = (size_t)G * kQPitch + 2 * kHeadDim;
  const size_t tiles = (size_t)kAttnTile * kKPitch * 2 + (size_t)kAttnTile * kHeadDim * 2;
  const size_t rest = (size_t)kAttnTile * G + 5 * (size_t)G + (size_t)G * kHeadDim;
  return attn_raw_bytes(G) + f32 * 4 + tiles + rest * 4 + 16;
}

// Loads cache rows [t0, t1) into the tile (none of them the new position).
__device__ __forceinline__ void load_tile(const AttnSmem& sm, const uint16_t* kc,
                                          const uint16_t* vc, int t0, int t1, int tid) {
  const int n = t1 - t0;
  for (int i = tid; i < n * 16; i += kAttnThreads) {  // 16 uint4 per row for K and V each
    const int r = i >> 4, c = i & 15;
    const uint4 kv = __ldcg(reinterpret_cast<const uint4*>(kc + (size_t)(t0 + r) * kHeadDim) + c);
    const uint4 vv = __ldcg(reinterpret_cast<const uint4*>(vc + (size_t)(t0 + r) * kHeadDim) + c);
    // K rows have an odd word pitch: store them word by word
    uint32_t* kd = reinterpret_cast<uint32_t*>(sm.kt_s + r * kKPitch) + 4 * c;
    kd[0] = kv.x;
    kd[1] = kv.y;
    kd[2] = kv.z;
    kd[3] = kv.w;
    *(reinterpret_cast<uint4*>(sm.vt_s + r * kHeadDim) + c) = vv;
  }
}

// Flash-decoding over this split's positions in tiles of kAttnTile: scores
// one thread per (position, head) from shared memory, online softmax per head,
// P.V one thread per dimension; the splits merge over DSMEM in rank order.
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const AttnParams p) {
  extern __shared__ __align__(16) unsigned char smem_attn[];
  const int G = p.group;
  const int kvh = blockIdx.x;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const AttnSmem sm = attn_layout(smem_attn, G);

  // The position and the cached rows below it were written by earlier steps:
  // load the first tile before waiting for this step's q/k/v.
  const int64_t raw_pos = *p.pos;
  // a position outside the cache is clamped (wrong output, never a wild store)
  const int pos = raw_pos < 0 ? 0 : (raw_pos >= p.max_seq ? p.max_seq - 1 : (int)raw_pos);
  const int P = pos + 1;
  const int chunk = (P + kAttnSplits - 1) / kAttnSplits;
  const int j0 = min(P, rank * chunk), j1 = min(P, j0 + chunk);
  const uint16_t* kc = p.k_cache + (size_t)kvh * p.max_seq * kHeadDim;
  const uint16_t* vc = p.v_cache + (size_t)kvh * p.max_seq * kHeadDim;
  load_tile(sm, kc, vc, j0, min(min(j1, j0 + kAttnTile), pos), tid);
  const float c = bf(p.cos_t[(size_t)pos * kHeadDim + tid]);
  const float s = bf(p.sin_t[(size_t)pos * kHeadDim + tid]);
  if (tid < G) {
    sm.hm_s[tid] = -INFINITY;
    sm.hl_s[tid] = 0.f;
  }

  grid_dependency_wait();  // qkv comes from the previous kernel
  {  // this group's q heads, k and v in one vectorised pass
    const uint4* q = reinterpret_cast<const uint4*>(p.qkv + (size_t)kvh * G * kHeadDim);
    const uint4* k = reinterpret_cast<const uint4*>(p.qkv + (size_t)(p.heads + kvh) * kHeadDim);
    const uint4* v =
        reinterpret_cast<const uint4*>(p.qkv + (size_t)(p.heads + p.kv_heads + kvh) * kHeadDim);
    uint4* dst = reinterpret_cast<uint4*>(sm.raw);
    for (int i = tid; i < (G + 2) * 16; i += kAttnThreads) {
      const int h = i >> 4, cc = i & 15;
      dst[i] = __ldcg((h < G ? q + h * 16 : (h == G ? k : v)) + cc);
    }
  }
  __syncthreads();
  for (int h = 0; h < G; ++h) sm.q_s[h * kQPitch + tid] = rope_dim(sm.raw + h * kHeadDim, tid, c, s);
  const float kr = rope_dim(sm.raw + G * kHeadDim, tid, c, s);
  const float vv = bf(sm.raw[(G + 1) * kHeadDim + tid]);
  sm.kn_s[tid] = kr;
  sm.vn_s[tid] = vv;
  if (pos >= j0 && pos < j1) {  // this split owns the new position: store it
    const size_t at = ((size_t)kvh * p.max_seq + pos) * kHeadDim + tid;
    p.k_cache[at] = to_bf(kr);
    p.v_cache[at] = to_bf(vv);
  }

  float o[16];  // o[h] for dimension tid
#pragma unroll
  for (int h = 0; h < 16; ++h) o[h] = 0.f;

  for (int t0 = j0; t0 < j1; t0 += kAttnTile) {
    const int t1 = min(j1, t0 + kAttnTile);
    if (t0 != j0) {
      __syncthreads();  // the previous tile is consumed
      load_tile(sm, kc, vc, t0, min(t1, pos), tid);
    }
    __syncthreads();
    const int n = t1 - t0;
    for (int pi = tid; pi < n * G; pi += kAttnThreads) {  // scores
      const int jl = pi / G, h = pi - jl * G;
      const float* qh = sm.q_s + h * kQPitch;
      float d = 0.f;
      if (t0 + jl == pos) {
        for (int e = 0; e < kHeadDim; ++e) d = fmaf(qh[e], sm.kn_s[e], d);
      } else {
        const uint32_t* kw = reinterpret_cast<const uint32_t*>(sm.kt_s + jl * kKPitch);
#pragma unroll 8
        for (int w = 0; w < kHeadDim / 2; ++w) {
          const uint32_t kk = kw[w];
          d = fmaf(qh[2 * w], bf(kk & 0xffffu), d);
          d = fmaf(qh[2 * w + 1], bf(kk >> 16), d);
        }
      }
      sm.sc_s[pi] = d * p.scale;
    }
    __syncthreads();
    for (int h = warp; h < G; h += kAttnThreads / 32) {  // online softmax per head
      float mx = -INFINITY;
      for (int jl = lane; jl < n; jl += 32) mx = fmaxf(mx, sm.sc_s[jl * G + h]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_old = sm.hm_s[h];
      const float m_new = fmaxf(m_old, mx);
      float sum = 0.f;
      for (int jl = lane; jl < n; jl += 32) {
        const float pr = __expf(sm.sc_s[jl * G + h] - m_new);
        sm.sc_s[jl * G + h] = pr;
        sum += pr;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      if (lane == 0) {
        const float alpha = (m_old == -INFINITY) ? 0.f : __expf(m_old - m_new);
        sm.ha_s[h] = alpha;
        sm.hl_s[h] = sm.hl_s[h] * alpha + sum;
        sm.hm_s[h] = m_new;
      }
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < 16; ++h)
      if (h < G) o[h] *= sm.ha_s[h];
    for (int jl = 0; jl < n; ++jl) {  // P.V, thread tid owns dimension tid
      const float vj = (t0 + jl == pos) ? sm.vn_s[tid] : bf(sm.vt_s[jl * kHeadDim + tid]);
#pragma unroll
      for (int h = 0; h < 16; ++h)
        if (h < G) o[h] = fmaf(sm.sc_s[jl * G + h], vj, o[h]);
    }
  }
  // this split's partial (an empty split leaves m = -inf, l = 0, o = 0)
#pragma unroll
  for (int h = 0; h < 16; ++h)
    if (h < G) sm.po_s[h * kHeadDim + tid] = o[h];
  if (tid < G) {
    sm.pm_s[tid] = sm.hm_s[tid];
    sm.pl_s[tid] = sm.hl_s[tid];
  }

  // Merge the splits of this KV head over DSMEM, in rank order.
  cluster.sync();
  // The next kernel (the o projection) may launch now. Triggering here, with
  // only the merge left, measured fastest for the whole step: earlier, its
  // CTAs contend with the tile loop; after the merge, its weight prefetch
  // starts too late.
  grid_launch_dependents();
  for (int idx = rank * kAttnThreads + tid; idx < G * kHeadDim; idx += kAttnThreads * kAttnSplits) {
    const int h = idx / kHeadDim;
    float M = -INFINITY;
    for (int r = 0; r < kAttnSplits; ++r) M = fmaxf(M, cluster.map_shared_rank(sm.pm_s, r)[h]);
    float L = 0.f, O = 0.f;
    for (int r = 0; r < kAttnSplits; ++r) {
      const float mr = cluster.map_shared_rank(sm.pm_s, r)[h];
      const float w = (mr == -INFINITY) ? 0.f : __expf(mr - M);
      L = fmaf(w, cluster.map_shared_rank(sm.pl_s, r)[h], L);
      O = fmaf(w, cluster.map_shared_rank(sm.po_s, r)[idx], O);
    }
    p.out[(size_t)(kvh * G + h) * kHeadDim + (idx - h * kHeadDim)] = to_bf(O / L);
  }
  cluster.sync();
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
  p.scale = 1.0f / sqrtf((float)kHeadDim);
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
// bulk copies; 8 consumer warps turn each stage's rows into logits.
constexpr int kLmConsumerWarps = 8;
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
