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

// Shared memory (floats): q[G][128], kn[128], vn[128], scores[chunk][G],
// warp partials wm[4][G], wl[4][G], wo[4][G][128], cluster partials
// pm[G], pl[G], po[G][128].
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const AttnParams p) {
  extern __shared__ float sm[];
  const int G = p.group;
  const int kvh = blockIdx.x;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  grid_dependency_wait();  // qkv comes from the previous kernel
  // a position outside the cache is clamped (wrong output, never a wild store)
  const int64_t raw_pos = *p.pos;
  const int pos = raw_pos < 0 ? 0 : (raw_pos >= p.max_seq ? p.max_seq - 1 : (int)raw_pos);
  const int P = pos + 1;
  const int chunk = (P + kAttnSplits - 1) / kAttnSplits;
  const int max_chunk = (p.max_seq + kAttnSplits - 1) / kAttnSplits;
  const int j0 = rank * chunk, j1 = min(P, j0 + chunk);

  float* q_s = sm;                       // [G][128]
  float* kn_s = q_s + G * kHeadDim;      // [128]
  float* vn_s = kn_s + kHeadDim;         // [128]
  float* sc_s = vn_s + kHeadDim;         // [max_chunk][G]
  float* wm_s = sc_s + max_chunk * G;    // [4][G]
  float* wl_s = wm_s + 4 * G;            // [4][G]
  float* wo_s = wl_s + 4 * G;            // [4][G][128]
  float* pm_s = wo_s + 4 * G * kHeadDim; // [G]
  float* pl_s = pm_s + G;                // [G]
  float* po_s = pl_s + G;                // [G][128]

  // RoPE on the group's q heads and on k; v as is.
  {
    const float c = bf(p.cos_t[(size_t)pos * kHeadDim + tid]);
    const float s = bf(p.sin_t[(size_t)pos * kHeadDim + tid]);
    for (int h = 0; h < G; ++h)
      q_s[h * kHeadDim + tid] = rope_dim(p.qkv + (size_t)(kvh * G + h) * kHeadDim, tid, c, s);
    const uint16_t* kh = p.qkv + (size_t)p.heads * kHeadDim + (size_t)kvh * kHeadDim;
    const uint16_t* vh = p.qkv + (size_t)(p.heads + p.kv_heads) * kHeadDim + (size_t)kvh * kHeadDim;
    const float kr = rope_dim(kh, tid, c, s);
    const float vv = bf(vh[tid]);
    kn_s[tid] = kr;
    vn_s[tid] = vv;
    if (pos >= j0 && pos < j1) {  // this CTA owns the new position: store it
      const size_t at = ((size_t)kvh * p.max_seq + pos) * kHeadDim + tid;
      p.k_cache[at] = to_bf(kr);
      p.v_cache[at] = to_bf(vv);
    }
  }
  __syncthreads();
  grid_launch_dependents();

  // Pass 1: scores s[j][h] = scale * q_h . k_j for this CTA's positions; warp
  // w takes positions j0 + w, j0 + w + 4, ...; lane owns dims 4*lane..+3.
  float wmax[16];
#pragma unroll
  for (int h = 0; h < 16; ++h) wmax[h] = -INFINITY;
  const uint16_t* kc = p.k_cache + (size_t)kvh * p.max_seq * kHeadDim;
  const uint16_t* vc = p.v_cache + (size_t)kvh * p.max_seq * kHeadDim;
  for (int j = j0 + warp; j < j1; j += 4) {
    float k4[4];
    if (j == pos) {
#pragma unroll
      for (int i = 0; i < 4; ++i) k4[i] = kn_s[4 * lane + i];
    } else {
      const uint2 kv = __ldcg(reinterpret_cast<const uint2*>(kc + (size_t)j * kHeadDim + 4 * lane));
      k4[0] = bf(kv.x & 0xffffu); k4[1] = bf(kv.x >> 16);
      k4[2] = bf(kv.y & 0xffffu); k4[3] = bf(kv.y >> 16);
    }
#pragma unroll
    for (int h = 0; h < 16; ++h) {
      if (h < G) {
        const float4 q4 = *reinterpret_cast<const float4*>(q_s + h * kHeadDim + 4 * lane);
        float d = q4.x * k4[0] + q4.y * k4[1] + q4.z * k4[2] + q4.w * k4[3];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
        d *= p.scale;
        if (lane == 0) sc_s[(j - j0) * G + h] = d;
        wmax[h] = fmaxf(wmax[h], d);
      }
    }
  }
  if (lane == 0) {
#pragma unroll
    for (int h = 0; h < 16; ++h)
      if (h < G) wm_s[warp * G + h] = wmax[h];
  }
  __syncthreads();

  // Pass 2: p = exp(s - m_h), l_h = sum p, o_h = sum p v_j.
  float m_h[16];
#pragma unroll
  for (int h = 0; h < 16; ++h)
    m_h[h] = (h < G) ? fmaxf(fmaxf(wm_s[h], wm_s[G + h]), fmaxf(wm_s[2 * G + h], wm_s[3 * G + h]))
                     : 0.f;
  float l_w[16], o_w[16][4];
#pragma unroll
  for (int h = 0; h < 16; ++h) {
    l_w[h] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) o_w[h][i] = 0.f;
  }
  for (int j = j0 + warp; j < j1; j += 4) {
    float v4[4];
    if (j == pos) {
#pragma unroll
      for (int i = 0; i < 4; ++i) v4[i] = vn_s[4 * lane + i];
    } else {
      const uint2 vv = __ldcg(reinterpret_cast<const uint2*>(vc + (size_t)j * kHeadDim + 4 * lane));
      v4[0] = bf(vv.x & 0xffffu); v4[1] = bf(vv.x >> 16);
      v4[2] = bf(vv.y & 0xffffu); v4[3] = bf(vv.y >> 16);
    }
#pragma unroll
    for (int h = 0; h < 16; ++h) {
      if (h < G) {
        const float pr = __expf(sc_s[(j - j0) * G + h] - m_h[h]);
        l_w[h] += pr;
#pragma unroll
        for (int i = 0; i < 4; ++i) o_w[h][i] = fmaf(pr, v4[i], o_w[h][i]);
      }
    }
  }
#pragma unroll
  for (int h = 0; h < 16; ++h) {
    if (h < G) {
      if (lane == 0) wl_s[warp * G + h] = l_w[h];
#pragma unroll
      for (int i = 0; i < 4; ++i) wo_s[(warp * G + h) * kHeadDim + 4 * lane + i] = o_w[h][i];
    }
  }
  __syncthreads();
  // CTA partial (all warps share m_h): fixed-order sum over the 4 warps.
#pragma unroll
  for (int h = 0; h < 16; ++h) {
    if (h >= G) break;
    po_s[h * kHeadDim + tid] = ((wo_s[(0 * G + h) * kHeadDim + tid] +
                                 wo_s[(1 * G + h) * kHeadDim + tid]) +
                                wo_s[(2 * G + h) * kHeadDim + tid]) +
                               wo_s[(3 * G + h) * kHeadDim + tid];
    if (tid == 0) {
      pm_s[h] = m_h[h];
      pl_s[h] = ((wl_s[h] + wl_s[G + h]) + wl_s[2 * G + h]) + wl_s[3 * G + h];
    }
  }

  // Merge the splits of this KV head over DSMEM, in rank order.
  cluster.sync();
  for (int idx = rank * kAttnThreads + tid; idx < G * kHeadDim; idx += kAttnThreads * kAttnSplits) {
    const int h = idx / kHeadDim;
    float M = -INFINITY;
    for (int r = 0; r < kAttnSplits; ++r) M = fmaxf(M, cluster.map_shared_rank(pm_s, r)[h]);
    float L = 0.f, O = 0.f;
    for (int r = 0; r < kAttnSplits; ++r) {
      const float mr = cluster.map_shared_rank(pm_s, r)[h];
      const float w = (mr == -INFINITY) ? 0.f : __expf(mr - M);
      L = fmaf(w, cluster.map_shared_rank(pl_s, r)[h], L);
      O = fmaf(w, cluster.map_shared_rank(po_s, r)[idx], O);
    }
    p.out[(size_t)(kvh * G + h) * kHeadDim + (idx - h * kHeadDim)] = to_bf(O / L);
  }
  cluster.sync();
}

static size_t attn_smem_bytes(int G, int max_seq) {
  const int max_chunk = (max_seq + kAttnSplits - 1) / kAttnSplits;
  return sizeof(float) * ((size_t)G * kHeadDim + 2 * kHeadDim + (size_t)max_chunk * G + 8 * G +
                          4 * (size_t)G * kHeadDim + 2 * G + (size_t)G * kHeadDim);
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
  const size_t smem = attn_smem_bytes(p.group, max_seq);
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

constexpr int kLmThreads = 256;

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

template <int CH>  // CH = hidden / 256: 16-byte chunks per lane per row
__global__ void __launch_bounds__(kLmThreads) lm_head_kernel(
    const uint16_t* __restrict__ h, const uint16_t* __restrict__ norm_w, float eps,
    const uint16_t* __restrict__ embed, int vocab, uint16_t* __restrict__ logits,
    int64_t* token, int64_t* pos, LmHeadWorkspace* ws) {
  constexpr int H = CH * 256;
  __shared__ float x_s[H];
  __shared__ float red[kLmThreads / 32];
  __shared__ unsigned long long best_s[kLmThreads / 32];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // Weights are constant: warm this CTA's first rows into L2 before waiting.
  grid_dependency_wait();
  // Final RMSNorm (fp32 normalisation, cast to bf16, times the bf16 weight).
  float ss = 0.f;
  for (int i = tid; i < H; i += kLmThreads) {
    const float v = bf(h[i]);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int w = 0; w < kLmThreads / 32; ++w) tot += red[w];
  const float inv = rsqrtf(tot / (float)H + eps);
  for (int i = tid; i < H; i += kLmThreads) x_s[i] = rbf(rbf(bf(h[i]) * inv) * bf(norm_w[i]));
  __syncthreads();
  grid_launch_dependents();

  // Lane l owns elements 8*(32*c + l) .. +7 of every row (coalesced 512 B per
  // warp load); x for them stays in registers.
  float xr[CH][8];
#pragma unroll
  for (int c = 0; c < CH; ++c)
#pragma unroll
    for (int i = 0; i < 8; ++i) xr[c][i] = x_s[8 * (32 * c + lane) + i];

  const int warps_total = gridDim.x * (kLmThreads / 32);
  const int gw = blockIdx.x * (kLmThreads / 32) + warp;
  unsigned long long best = 0;
  // two rows per warp iteration: 2*CH independent 16-byte loads in flight
  for (int r = 2 * gw; r < vocab; r += 2 * warps_total) {
    const int r1 = min(r + 1, vocab - 1);
    uint4 a[CH], b[CH];
    const uint4* ra = reinterpret_cast<const uint4*>(embed + (size_t)r * H);
    const uint4* rb = reinterpret_cast<const uint4*>(embed + (size_t)r1 * H);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      a[c] = __ldcs(ra + 32 * c + lane);
      b[c] = __ldcs(rb + 32 * c + lane);
    }
    float da = 0.f, db = 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const uint32_t* av = reinterpret_cast<const uint32_t*>(&a[c]);
      const uint32_t* bv = reinterpret_cast<const uint32_t*>(&b[c]);
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
      const uint16_t la = to_bf(da), lb = to_bf(db);
      if (logits) {
        logits[r] = la;
        if (r + 1 < vocab) logits[r + 1] = lb;
      }
      const unsigned long long ka =
          ((unsigned long long)order_key(bf(la)) << 32) | (0xffffffffu - (uint32_t)r);
      best = ka > best ? ka : best;
      if (r + 1 < vocab) {
        const unsigned long long kb =
            ((unsigned long long)order_key(bf(lb)) << 32) | (0xffffffffu - (uint32_t)(r + 1));
        best = kb > best ? kb : best;
      }
    }
  }
  if (lane == 0) best_s[warp] = best;
  __syncthreads();
  if (tid == 0) {
    unsigned long long b = 0;
    for (int w = 0; w < kLmThreads / 32; ++w) b = best_s[w] > b ? best_s[w] : b;
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
  const int sms = device_info(dev).sm_count > 0 ? device_info(dev).sm_count : 148;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * sms));
  cfg.blockDim = dim3(kLmThreads);
  cfg.stream = stream;
  cudaLaunchAttribute at = pdl_attr(pdl);
  cfg.attrs = &at;
  cfg.numAttrs = 1;
  const uint16_t* hh = static_cast<const uint16_t*>(h);
  const uint16_t* nw = static_cast<const uint16_t*>(norm_w);
  const uint16_t* em = static_cast<const uint16_t*>(embed);
  uint16_t* lg = static_cast<uint16_t*>(logits);
  LmHeadWorkspace* ws = static_cast<LmHeadWorkspace*>(workspace);
  cudaError_t e;
  switch (hidden / 256) {
    case 1: e = cudaLaunchKernelEx(&cfg, lm_head_kernel<1>, hh, nw, eps, em, vocab, lg, token, pos, ws); break;
    case 2: e = cudaLaunchKernelEx(&cfg, lm_head_kernel<2>, hh, nw, eps, em, vocab, lg, token, pos, ws); break;
    case 4: e = cudaLaunchKernelEx(&cfg, lm_head_kernel<4>, hh, nw, eps, em, vocab, lg, token, pos, ws); break;
    case 6: e = cudaLaunchKernelEx(&cfg, lm_head_kernel<6>, hh, nw, eps, em, vocab, lg, token, pos, ws); break;
    case 8: e = cudaLaunchKernelEx(&cfg, lm_head_kernel<8>, hh, nw, eps, em, vocab, lg, token, pos, ws); break;
    case 16: e = cudaLaunchKernelEx(&cfg, lm_head_kernel<16>, hh, nw, eps, em, vocab, lg, token, pos, ws); break;
    default: return fail(W4_ERR_UNSUPPORTED, "w4_lm_head_argmax: hidden %d not in {256, 512, 1024, 1536, 2048, 4096}", hidden);
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
constexpr size_t kStaticScratchBytes = 256;
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
  const size_t smem = attn_smem_bytes(16, 16384);
  cudaError_t e = cudaFuncSetAttribute(attention_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)std::min<size_t>(smem, (size_t)di.max_smem_optin));
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(attention smem)");
  return W4_OK;
}

}  // namespace w4
