// w4_gemv.cu - host side of the fused W4A16 GEMV (tile choice, tensor maps,
// launch) and its plain instances; the kernel is in w4_gemv_kernel.cuh.
#include "w4_gemv_kernel.cuh"

#include <algorithm>
#include <new>

namespace w4 {

void* gemv_kernel_plain(int bf16, int mb, int sw, int rg) {
  if (bf16)
    return mb == 1 ? gemv_pick_tile<true, 1, kOpsPlain>(sw, rg)
                   : gemv_pick_tile<true, 2, kOpsPlain>(sw, rg);
  return mb == 1 ? gemv_pick_tile<false, 1, kOpsPlain>(sw, rg)
                 : gemv_pick_tile<false, 2, kOpsPlain>(sw, rg);
}

namespace {

// The instance a launch uses: plain (one or several tiles per CTA column),
// plain with the gathered output, the fused decode combination it matches
// (bf16 activations, up to 8 batch rows), or the generic one.
void* pick_kernel(int bf16, int mb, int sw, int rg, int ops, bool tiles) {
  if (ops == kOpsPeer && !tiles) return gemv_kernel_peer(bf16, mb, sw, rg);
  if (ops == kOpsPeer) return gemv_kernel_generic(bf16, mb, sw, rg);
  if (ops == kOpsPlain)
    return tiles ? gemv_kernel_plain_tiles(bf16, mb, sw, rg) : gemv_kernel_plain(bf16, mb, sw, rg);
  if (tiles) return gemv_kernel_generic(bf16, mb, sw, rg);
  if (ops >= kOpsFusedFirst && ops <= kOpsFusedLast && bf16 && mb == 1)
    return gemv_kernel_fused(ops, sw, rg);
  return gemv_kernel_generic(bf16, mb, sw, rg);
}

constexpr int kSW[] = {1, 2, 4};

}  // namespace

int gemv_tiles(int N, const w4_gemv_config& c) {
  const int nt = 32 * c.strips;
  return (N + nt - 1) / nt;
}

int gemv_columns(int N, const w4_gemv_config& c) {
  const int t = gemv_tiles(N, c);
  return (c.columns > 0 && c.columns < t) ? c.columns : t;
}

size_t gemv_smem_bytes(int M, int K, int N, const w4_gemv_config& c) {
  const int groups = K / 128;
  const int cols = gemv_columns(N, c);
  const size_t tiles_per_cta = (gemv_tiles(N, c) + cols - 1) / cols;
  const int gps = (groups + c.split - 1) / c.split;
  const size_t nt = 32 * (size_t)c.strips;
  const size_t stage = (size_t)c.strips * c.row_groups * 16 * 128;
  const size_t scale = ((size_t)c.row_groups * nt * 2 + 127) / 128 * 128;
  const size_t plane = (size_t)gps * 16 * 16 + 16;
  // beta and 2^-e per (row, group), then 1/rms per row
  const size_t beta = (((size_t)M * gps + 3) & ~(size_t)3) * 4 * 2 + 16 * 4;
  const size_t tile = (size_t)M * nt * 4;
  return 1024 + c.stages * (stage + scale) + M * plane + beta +
         tiles_per_cta * c.row_groups * tile + tile /* epilogue operands */ + 2 * c.stages * sizeof(uint64_t) + 16;  // + the epoch word
}

int gemv_validate_config(int M, int K, int N, const w4_gemv_config& c, const DeviceInfo& di) {
  if (c.strips < 1 || c.row_groups < 1)
    return fail(W4_ERR_INVALID_ARG, "unsupported tile strips=%d row_groups=%d", c.strips,
                c.row_groups);
  const bool several = gemv_columns(N, c) < gemv_tiles(N, c);
  if (!gemv_kernel_plain(0, 1, c.strips, c.row_groups) &&
      !(several && gemv_kernel_plain_tiles(0, 1, c.strips, c.row_groups)))
    return fail(W4_ERR_INVALID_ARG,
                "unsupported tile strips=%d row_groups=%d (16 compute warps need fewer CTA "
                "columns than tiles)",
                c.strips, c.row_groups);
  if (c.stages < 2 || c.stages > 8)
    return fail(W4_ERR_INVALID_ARG, "stages=%d outside 2..8", c.stages);
  if (c.split < 1 || c.split > 16)
    return fail(W4_ERR_INVALID_ARG, "split=%d outside 1..16", c.split);
  if (c.split > K / 128)
    return fail(W4_ERR_INVALID_ARG, "split=%d exceeds the %d K groups", c.split, K / 128);
  if (c.columns < 0) return fail(W4_ERR_INVALID_ARG, "columns=%d is negative", c.columns);
  const size_t smem = gemv_smem_bytes(M, K, N, c);
  if (smem > (size_t)di.max_smem_optin)
    return fail(W4_ERR_UNSUPPORTED,
                "tile needs %zu B of shared memory (device allows %d); raise split", smem,
                di.max_smem_optin);
  return W4_OK;
}

int gemv_choose_config(int M, int K, int N, int split_k, int num_warps, const DeviceInfo& di,
                       w4_gemv_config* out) {
  const int groups = K / 128;
  const int sms = di.sm_count > 0 ? di.sm_count : 148;
  const int cw = (num_warps == 4) ? 4 : 8;
  // The widest strips that still leave at least 1.5 column tiles per SM: a
  // wide tile streams longer row segments, but a grid that does not fill the
  // GPU costs more (tuned tables: one 32-column strip with 8 row groups wins
  // on every decode-sized shape, 2-4 strips only once N is large).
  int sw = 1;
  for (int c : {4, 2}) {
    const int t = (N + 32 * c - 1) / (32 * c);
    if (cw / c >= 1 && 32 * c <= N && 2 * t >= 3 * sms) {
      sw = c;
      break;
    }
  }
  const int rg = std::max(1, cw / sw);
  const int tiles = (N + 32 * sw - 1) / (32 * sw);
  int split = split_k;
  if (split <= 0) {
    // Split K only when the column tiles do not fill the GPU: towards about
    // 2.5 CTAs per SM, keeping at least RG groups per split.
    split = 1;
    if (2 * tiles < 3 * sms)
      split = std::max(1, std::min({(5 * sms + 2 * tiles - 1) / (2 * tiles), 8,
                                    std::max(1, groups / rg)}));
  }
  w4_gemv_config c{sw, rg, 4, split, 0};
  const int gps = (groups + split - 1) / split;
  const int stages_needed = (gps + rg - 1) / rg;
  // Keep the whole share in flight when it is small (each stage that waits
  // for a free slot costs a DRAM round trip); 6 slots suffice for streaming.
  c.stages = std::max(2, std::min(6, stages_needed));
  while (c.stages > 2 && gemv_smem_bytes(M, K, N, c) > (size_t)di.max_smem_optin / 2) --c.stages;
  // Grow the split until the activation slice fits in shared memory.
  while (gemv_smem_bytes(M, K, N, c) > (size_t)di.max_smem_optin && c.split < 16 &&
         c.split < groups && split_k <= 0)
    ++c.split;
  // Very large N (the vocab projection): a streaming grid of one 16-warp CTA
  // per SM, each taking its column tiles round-robin (tuned on 8192 x 128256:
  // 82.4 us against 89.9 for the best one-tile-per-CTA grid)
  if (M <= 8 && split_k <= 0 && num_warps <= 0 && N >= 4 * 128 * sms) {
    const w4_gemv_config s{4, 4, 4, 1, 0, sms};
    if (gemv_smem_bytes(M, K, N, s) <= (size_t)di.max_smem_optin) c = s;
  }
  *out = c;
  return gemv_validate_config(M, K, N, c, di);
}

// An encoded tensor map is a pure function of the arguments below, so the
// maps of recent launches are kept per host thread and reused when every
// argument matches (a decode loop launches the same weights every step; an
// encode costs about a microsecond of host time).
struct MapKey {
  const void* base;
  uint64_t cols, rows;
  uint32_t box_cols, box_rows;
  int dt, elem_bytes, swz;
  bool operator==(const MapKey& o) const {
    return base == o.base && cols == o.cols && rows == o.rows && box_cols == o.box_cols &&
           box_rows == o.box_rows && dt == o.dt && elem_bytes == o.elem_bytes && swz == o.swz;
  }
};
struct MapSlot {
  MapKey key;
  CUtensorMap map;
  bool valid;
};
constexpr int kMapSlots = 64;
static thread_local MapSlot t_map_cache[kMapSlots];

static bool make_map(CUtensorMap* map, CUtensorMapDataType dt, int elem_bytes, const void* base,
                     uint64_t cols, uint64_t rows, uint32_t box_cols, uint32_t box_rows,
                     CUtensorMapSwizzle swz) {
  const MapKey key{base, cols, rows, box_cols, box_rows, (int)dt, elem_bytes, (int)swz};
  const uint64_t h = (reinterpret_cast<uintptr_t>(base) >> 8) ^ (cols * 0x9E3779B1u) ^
                     (rows << 7) ^ ((uint64_t)box_cols << 17) ^ ((uint64_t)box_rows << 23) ^
                     ((uint64_t)dt << 29);
  MapSlot& slot = t_map_cache[(h ^ (h >> 17)) % kMapSlots];
  if (slot.valid && slot.key == key) {
    *map = slot.map;
    return true;
  }
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  slot.key = key;
  slot.map = *map;
  slot.valid = true;
  return true;
}

static int gemv_kernel_attributes(void* k, const DeviceInfo& di);

int gemv_init_device(const DeviceInfo& di) {
  for (int sw : kSW)
    for (int rg = 1; rg <= 8; rg *= 2) {
      if (!gemv_kernel_plain_tiles(0, 1, sw, rg)) continue;
      for (int b = 0; b < 2; ++b)
        for (int mb = 1; mb <= 2; ++mb)
          for (void* k : {gemv_kernel_plain(b, mb, sw, rg), gemv_kernel_generic(b, mb, sw, rg),
                          gemv_kernel_plain_tiles(b, mb, sw, rg), gemv_kernel_peer(b, mb, sw, rg)}) {
            if (!k) continue;  // the 16-warp tiles exist as plain-tiles instances only
            const int st = gemv_kernel_attributes(k, di);
            if (st != W4_OK) return st;
          }
      for (int ops = kOpsFusedFirst; ops <= kOpsFusedLast; ++ops) {
        void* k = gemv_kernel_fused(ops, sw, rg);
        if (!k) continue;
        const int st = gemv_kernel_attributes(k, di);
        if (st != W4_OK) return st;
      }
    }
  return W4_OK;
}

// Shared-memory limit, non-portable clusters and the carveout of one instance.
static int gemv_kernel_attributes(void* k, const DeviceInfo& di) {
  cudaError_t e =
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, di.max_smem_optin);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max smem)");
  e = cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(cluster)");
  // One carveout for every kernel of the library: CTAs of a dependent
  // (PDL) grid can then share SMs with the grid still finishing.
  e = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(carveout)");
  return W4_OK;
}

// Everything a launch needs except x, y and the stream: the instance, its
// encoded tensor maps, the kernel parameters and the launch geometry.
struct GemvPrepared {
  CUtensorMap tm_w, tm_s;
  GemvParams p;
  PeerParams pp;
  void* kfn;
  dim3 grid, block;
  size_t smem;
  cudaLaunchAttribute attrs[2];
  int num_attrs;
  int device;
};

static int gemv_prepare(const GemvLaunch& L, GemvPrepared* g) {
  int dev = 0;
  int st = current_device(&dev);
  if (st != W4_OK) return st;
  const DeviceInfo& di = device_info(dev);
  const w4_gemv_config& c = L.cfg;
  st = gemv_validate_config(L.M, L.K, L.N, c, di);
  if (st != W4_OK) return st;
  const int tiles = gemv_tiles(L.N, c);
  const int columns = gemv_columns(L.N, c);
  if (columns < tiles && (L.ops.epilogue != W4_EPI_NONE || L.peer))
    return fail(W4_ERR_UNSUPPORTED,
                "columns=%d below the %d column tiles needs no epilogue and a local output",
                columns, tiles);

  const int mb = L.M > 8 ? 2 : 1;
  const int plain_ops = ops_for(L.ops.prologue, L.ops.epilogue);
  const int ops = !L.peer ? plain_ops : plain_ops == kOpsPlain ? kOpsPeer : kOpsGeneric;
  g->kfn = pick_kernel(L.x_bf16, mb, c.strips, c.row_groups, ops, columns < tiles);
  if (!g->kfn)
    return fail(W4_ERR_UNSUPPORTED, "tile strips=%d row_groups=%d has no instance with a prologue",
                c.strips, c.row_groups);
  const int nt = 32 * c.strips;
  const int rows = L.K / 8;

  if (!make_map(&g->tm_w, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, L.packed, (uint64_t)L.N,
                (uint64_t)rows, 32, (uint32_t)(c.row_groups * 16), CU_TENSOR_MAP_SWIZZLE_128B))
    return fail(W4_ERR_CUDA, "cuTensorMapEncodeTiled failed for packed [%d, %d]", rows, L.N);
  if (!make_map(&g->tm_s, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, L.scales, (uint64_t)L.N,
                (uint64_t)(L.K / 128), (uint32_t)nt, (uint32_t)c.row_groups,
                CU_TENSOR_MAP_SWIZZLE_NONE))
    return fail(W4_ERR_CUDA, "cuTensorMapEncodeTiled failed for scales [%d, %d]", L.K / 128,
                L.N);

  GemvParams& p = g->p;
  p.x = L.x;
  p.y = L.y;
  p.M = L.M;
  p.K = L.K;
  p.N = L.N;
  p.groups_total = L.K / 128;
  p.groups_per_split = (p.groups_total + c.split - 1) / c.split;
  p.n_tiles = tiles;
  p.tiles_per_cta = (tiles + columns - 1) / columns;
  p.stages = c.stages;
  p.y_bf16 = L.y_bf16;
  p.err = di.err_word;
  p.pro = L.ops.prologue;
  p.pro_w = L.ops.norm_weight;
  p.eps = L.ops.eps;
  p.epi = L.ops.epilogue;
  p.epi_src = L.ops.epi_src;

  g->grid = dim3((unsigned)columns, (unsigned)c.split, 1);
  g->block = dim3((unsigned)((c.strips * c.row_groups + 1) * 32), 1, 1);
  g->smem = gemv_smem_bytes(L.M, L.K, L.N, c);
  int na = 0;
  if (c.split > 1) {
    g->attrs[na].id = cudaLaunchAttributeClusterDimension;
    g->attrs[na].val.clusterDim.x = 1;
    g->attrs[na].val.clusterDim.y = (unsigned)c.split;
    g->attrs[na].val.clusterDim.z = 1;
    ++na;
  }
  if (c.pdl) {
    g->attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    g->attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  g->num_attrs = na;
  g->pp = PeerParams{};
  if (L.peer) {
    const w4_peer_out& po = *L.peer;
    PeerParams& pp = g->pp;
    pp.world = po.world;
    pp.rank = po.rank;
    pp.n_full = po.n_full;
    pp.col_off = po.col_off;
    for (int b = 0; b < 2; ++b)
      for (int q = 0; q < W4B200_MAX_PEERS; ++q) pp.y[b][q] = po.y[b][q];
    for (int q = 0; q < W4B200_MAX_PEERS; ++q) pp.flags[q] = po.flags[q];
    pp.state = po.state;
  }
  g->device = dev;
  return W4_OK;
}

// Launches a prepared GEMV on x and y (the prepared parameters are copied:
// concurrent launches of one plan from several host threads are safe).
static int gemv_launch_prepared(const GemvPrepared& g, const void* x, void* y,
                                cudaStream_t stream) {
  GemvParams p = g.p;
  p.x = x;
  p.y = y;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = g.grid;
  cfg.blockDim = g.block;
  cfg.dynamicSmemBytes = g.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2] = {g.attrs[0], g.attrs[1]};
  cfg.attrs = attrs;
  cfg.numAttrs = (unsigned)g.num_attrs;
  PeerParams pp = g.pp;
  CUtensorMap tm_w = g.tm_w, tm_s = g.tm_s;
  void* args[] = {&tm_w, &tm_s, &p, &pp};
  cudaError_t e = cudaLaunchKernelExC(&cfg, g.kfn, args);
  if (e != cudaSuccess) return cuda_fail(e, "w4_gemv launch");
  return W4_OK;
}

int launch_gemv(const GemvLaunch& L, cudaStream_t stream) {
  GemvPrepared g;
  const int st = gemv_prepare(L, &g);
  if (st != W4_OK) return st;
  return gemv_launch_prepared(g, L.x, L.y, stream);
}

// ---------------------------------------------------------------- plans

struct GemvPlan {
  GemvPrepared g;
  size_t x_bytes, y_bytes;
};

int gemv_plan_create(const GemvLaunch& L, void** out) {
  GemvPlan* plan = new (std::nothrow) GemvPlan;
  if (!plan) return fail(W4_ERR_INVALID_ARG, "w4_gemv_plan_create: out of host memory");
  const int st = gemv_prepare(L, &plan->g);
  if (st != W4_OK) {
    delete plan;
    return st;
  }
  plan->x_bytes = (size_t)L.M * L.K * 2;
  plan->y_bytes = (size_t)L.M * L.N * 2;
  *out = plan;
  return W4_OK;
}

int gemv_plan_launch(const void* handle, const void* x_host, void* x, void* y, void* y_host,
                     cudaStream_t stream) {
  const GemvPlan& plan = *static_cast<const GemvPlan*>(handle);
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev != plan.g.device)
    return fail(W4_ERR_INVALID_ARG, "w4_gemv_plan: made on device %d, called on device %d",
                plan.g.device, dev);
  if (x_host && (e = cudaMemcpyAsync(x, x_host, plan.x_bytes, cudaMemcpyHostToDevice, stream)) !=
                    cudaSuccess)
    return cuda_fail(e, "w4_gemv_plan: copy of x to the device");
  int st = gemv_launch_prepared(plan.g, x, y, stream);
  if (st != W4_OK) return st;
  if (y_host && (e = cudaMemcpyAsync(y_host, y, plan.y_bytes, cudaMemcpyDeviceToHost, stream)) !=
                    cudaSuccess)
    return cuda_fail(e, "w4_gemv_plan: copy of y to the host");
  return W4_OK;
}

int gemv_plans_launch(const void* const* handles, int n, const void* x_host, void* x, void* y,
                      void* y_host, cudaStream_t stream) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  size_t x_total = 0, y_total = 0;
  for (int i = 0; i < n; ++i) {
    const GemvPlan& plan = *static_cast<const GemvPlan*>(handles[i]);
    if (plan.g.device != dev)
      return fail(W4_ERR_INVALID_ARG, "w4_gemv_plans: plan %d made on device %d, called on %d",
                  i, plan.g.device, dev);
    x_total += plan.x_bytes;
    y_total += plan.y_bytes;
  }
  if (x_host && (e = cudaMemcpyAsync(x, x_host, x_total, cudaMemcpyHostToDevice, stream)) !=
                    cudaSuccess)
    return cuda_fail(e, "w4_gemv_plans: copy of x to the device");
  size_t xo = 0, yo = 0;
  for (int i = 0; i < n; ++i) {
    const GemvPlan& plan = *static_cast<const GemvPlan*>(handles[i]);
    const int st = gemv_launch_prepared(plan.g, static_cast<const char*>(x) + xo,
                                        static_cast<char*>(y) + yo, stream);
    if (st != W4_OK) return st;
    xo += plan.x_bytes;
    yo += plan.y_bytes;
  }
  if (y_host && (e = cudaMemcpyAsync(y_host, y, y_total, cudaMemcpyDeviceToHost, stream)) !=
                    cudaSuccess)
    return cuda_fail(e, "w4_gemv_plans: copy of y to the host");
  return W4_OK;
}

void gemv_plan_destroy(void* handle) { delete static_cast<GemvPlan*>(handle); }

}  // namespace w4
