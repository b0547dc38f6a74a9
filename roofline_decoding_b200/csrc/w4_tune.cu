// w4_tune.cu - per-shape tile tuner of the fused GEMV for C / C++ hosts.
//
// Replaces the reference's _tune_num_warps (roofline/kernels.py:211-247),
// which timed num_warps {4, 8} with a fresh zeroed output per trial because
// its split-K accumulated with atomics. The GEMV here writes without atomics,
// so trials share buffers. What matters instead: B200's 126 MB L2 would hold
// any decode-sized weight matrix, and a lone microsecond launch cannot be timed
// with events. So every candidate tile is timed as one CUDA graph of dependent
// (PDL) launches, each on its own copy of random weights, the copies together
// exceeding 3x L2 - the way the GEMVs of a decode step run. The candidate set
// and the timing are those of roofline_decoding_b200/tuner.py.
#include "w4_internal.h"

#include <cuda_fp16.h>

#include <algorithm>
#include <vector>

namespace w4 {

namespace {

// Deterministic pseudo-random words (a 64-bit mix of the index and seed).
__device__ __forceinline__ uint32_t mix32(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return (uint32_t)((z ^ (z >> 31)) >> 16);
}

__global__ void fill_words(uint32_t* p, size_t n, uint64_t seed) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    p[i] = mix32(seed * 0x100000001B3ull + i);
}

// Halves in [lo, lo + span): scales (fp16) or activations (fp16 / bf16 bits).
__global__ void fill_halves(uint16_t* p, size_t n, uint64_t seed, float lo, float span, int bf16) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const float v = lo + span * (float)(mix32(seed * 0x100000001B3ull + i) & 0xFFFF) / 65536.f;
    p[i] = bf16 ? (uint16_t)(__float_as_uint(v) >> 16) : __half_as_ushort(__float2half_rn(v));
  }
}

// Candidate tiles: the tuner's search space (strips x compute warps x split x
// stages, splits only while the grid would not already have plenty of CTAs)
// plus the library's default choice.
std::vector<w4_gemv_config> candidates(int M, int K, int N, int split_k, int num_warps, int sms,
                                       const DeviceInfo& di) {
  const int groups = K / 128;
  // 16 compute warps: the streaming tiles (one CTA per SM, several column
  // tiles per CTA column) only
  std::vector<int> warps =
      num_warps > 0 ? std::vector<int>{num_warps} : std::vector<int>{4, 8, 16};
  std::vector<int> splits;
  if (split_k > 0) {
    splits.push_back(split_k);
  } else {
    for (int s : {1, 2, 3, 4, 6, 8, 12, 16})
      if (s <= groups) splits.push_back(s);
  }
  std::vector<w4_gemv_config> out;
  auto add = [&](const w4_gemv_config& c) {
    for (const w4_gemv_config& o : out)
      if (o.strips == c.strips && o.row_groups == c.row_groups && o.stages == c.stages &&
          o.split == c.split && o.columns == c.columns)
        return;
    out.push_back(c);
  };
  for (int cw : warps)
    for (int strips : {1, 2, 4}) {
      const int rg = cw / strips;
      if (rg != 1 && rg != 2 && rg != 4 && rg != 8) continue;
      if (cw == 16 && strips == 1) continue;
      if (strips > 1 && 32 * strips > N) continue;
      const int tiles = (N + 32 * strips - 1) / (32 * strips);
      for (int split : splits) {
        // one CTA per column tile (0), and for large N grids of one or two
        // CTAs per SM in all, each CTA column streaming two or more tiles
        // ... and the column counts that give every CTA column the same
        // number of tiles (2..8) with 0.6 to 2 CTAs per SM
        int col_opts[11] = {0};
        int n_col = 1;
        auto add_col = [&](int c) {
          for (int i = 0; i < n_col; ++i)
            if (col_opts[i] == c) return;
          col_opts[n_col++] = c;
        };
        for (int per_sm = 1; per_sm <= 2; ++per_sm) {
          const int c = std::max(1, (per_sm * sms + split / 2) / split);
          if (2 * c <= tiles) add_col(c);
        }
        for (int t = 2; t <= 8; ++t) {
          const int c = tiles / t;
          if (tiles % t == 0 && 10 * c * split >= 6 * sms && c * split <= 2 * sms) add_col(c);
        }
        for (int ci = 0; ci < n_col; ++ci) {
          const int columns = col_opts[ci];
          if (cw == 16 && (columns == 0 || columns * split > sms + split)) continue;
          const int ctas = (columns ? columns : tiles) * split;
          if (split_k <= 0 && split > 1 && ctas > 6 * sms) continue;
          const int gps = (groups + split - 1) / split;
          const int per_col = columns ? (tiles + columns - 1) / columns : 1;
          const int n_stages = (gps + rg - 1) / rg * per_col;
          for (int stages : {2, 3, 4, 5, 6, 8}) {
            if (stages > std::max(2, n_stages)) continue;
            if (columns && ((stages != 4 && stages != 6) ||
                            (split != 1 && split != 2 && split != 4 && split != 8)))
              continue;  // a streaming ring: fewer depths to try
            add(w4_gemv_config{strips, rg, stages, split, 0, columns});
          }
        }
      }
    }
  w4_gemv_config d{};
  if (gemv_choose_config(M, K, N, split_k, num_warps, di, &d) == W4_OK) add(d);
  return out;
}

struct Buffers {
  std::vector<void*> ptrs;
  ~Buffers() {
    for (void* p : ptrs) cudaFree(p);
  }
  void* alloc(size_t bytes) {
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
    ptrs.push_back(p);
    return p;
  }
};

// Mean per-launch time (us) of a graph of `copies` dependent launches of cfg,
// best of 3 replays; negative if the tile cannot be launched.
float time_candidate(const GemvLaunch& base, const w4_gemv_config& cfg,
                     const std::vector<const int32_t*>& packed,
                     const std::vector<const void*>& scales, cudaStream_t s) {
  GemvLaunch L = base;
  L.cfg = cfg;
  L.cfg.pdl = 1;
  L.packed = packed[0];
  L.scales = scales[0];
  if (launch_gemv(L, s) != W4_OK || cudaStreamSynchronize(s) != cudaSuccess) return -1.f;
  cudaGraph_t graph = nullptr;
  if (cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return -1.f;
  bool ok = true;
  for (size_t i = 0; i < packed.size() && ok; ++i) {
    L.packed = packed[i];
    L.scales = scales[i];
    ok = launch_gemv(L, s) == W4_OK;
  }
  const cudaError_t ec = cudaStreamEndCapture(s, &graph);
  if (!ok || ec != cudaSuccess || !graph) {
    if (graph) cudaGraphDestroy(graph);
    return -1.f;
  }
  cudaGraphExec_t exec = nullptr;
  float best = -1.f;
  if (cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess) {
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    cudaGraphLaunch(exec, s);  // upload
    for (int rep = 0; rep < 3; ++rep) {
      cudaEventRecord(a, s);
      cudaGraphLaunch(exec, s);
      cudaEventRecord(b, s);
      if (cudaEventSynchronize(b) != cudaSuccess) {
        best = -1.f;
        break;
      }
      float ms = 0.f;
      cudaEventElapsedTime(&ms, a, b);
      const float us = ms * 1e3f / (float)packed.size();
      best = (best < 0.f) ? us : std::min(best, us);
    }
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    cudaGraphExecDestroy(exec);
  }
  cudaGraphDestroy(graph);
  return best;
}

}  // namespace

int gemv_tune(int M, int K, int N, int x_bf16, int y_bf16, int split_k, int num_warps,
              w4_gemv_config* out, float* best_us) {
  int dev = 0;
  int st = current_device(&dev);
  if (st != W4_OK) return st;
  const DeviceInfo& di = device_info(dev);
  int l2 = 0;
  cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, dev);
  const size_t pw = (size_t)(K / 8) * N * 4, sw = (size_t)(K / 128) * N * 2;
  const size_t per_copy = pw + sw;
  const int copies = (int)std::min<size_t>(
      256, std::max<size_t>(8, (3 * (size_t)l2 + per_copy - 1) / per_copy));

  Buffers buf;
  std::vector<const int32_t*> packed(copies);
  std::vector<const void*> scales(copies);
  void* x = buf.alloc((size_t)M * K * 2);
  void* y = buf.alloc((size_t)M * N * 2);
  if (!x || !y) return fail(W4_ERR_CUDA, "w4_gemv_tune: cudaMalloc failed");
  fill_halves<<<148, 256>>>(static_cast<uint16_t*>(x), (size_t)M * K, 7, -1.f, 2.f, x_bf16);
  for (int i = 0; i < copies; ++i) {
    void* p = buf.alloc(pw);
    void* s = buf.alloc(sw);
    if (!p || !s)
      return fail(W4_ERR_CUDA, "w4_gemv_tune: cudaMalloc of %d weight copies failed", copies);
    fill_words<<<148 * 4, 256>>>(static_cast<uint32_t*>(p), pw / 4, 1000 + i);
    fill_halves<<<148, 256>>>(static_cast<uint16_t*>(s), sw / 2, 2000 + i, 1e-3f, 1e-2f, 0);
    packed[i] = static_cast<const int32_t*>(p);
    scales[i] = s;
  }
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "w4_gemv_tune fill");

  cudaStream_t s = nullptr;
  if ((e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking)) != cudaSuccess)
    return cuda_fail(e, "w4_gemv_tune stream");
  GemvLaunch base{};
  base.x = x;
  base.y = y;
  base.x_bf16 = x_bf16;
  base.y_bf16 = y_bf16;
  base.M = M;
  base.K = K;
  base.N = N;
  const std::vector<w4_gemv_config> cands =
      candidates(M, K, N, split_k, num_warps, di.sm_count > 0 ? di.sm_count : 148, di);
  float best = -1.f;
  w4_gemv_config best_c{};
  for (const w4_gemv_config& c : cands) {
    if (gemv_validate_config(M, K, N, c, di) != W4_OK) continue;  // does not fit
    const float us = time_candidate(base, c, packed, scales, s);
    if (us > 0.f && (best < 0.f || us < best)) {
      best = us;
      best_c = c;
    }
  }
  cudaStreamDestroy(s);
  if (best < 0.f) return fail(W4_ERR_UNSUPPORTED, "w4_gemv_tune: no tile could be launched");
  best_c.pdl = 0;
  *out = best_c;
  if (best_us) *best_us = best;
  return W4_OK;
}

}  // namespace w4
