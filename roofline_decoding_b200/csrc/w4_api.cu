// w4_api.cu - extern "C" entry points of libw4b200.so (declared in
// include/w4b200.h): argument validation, one-off device set-up and dispatch.
#include "w4_internal.h"

#include <cstring>

#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

namespace w4 {

namespace {
thread_local std::string g_last_error;
std::mutex g_init_mutex;
constexpr int kMaxDevices = 64;
DeviceInfo g_devices[kMaxDevices];
bool g_ready[kMaxDevices] = {};
EncodeTiledFn g_encode = nullptr;

__device__ int g_error_word = 0;
}  // namespace

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(W4_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

const DeviceInfo& device_info(int device) { return g_devices[device]; }
EncodeTiledFn encode_tiled_fn() { return g_encode; }

int current_device(int* dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (*dev < 0 || *dev >= kMaxDevices) return fail(W4_ERR_UNSUPPORTED, "device %d", *dev);
  if (!g_ready[*dev]) return w4_init(*dev);
  return W4_OK;
}

namespace {

int init_locked(int device) {
  if (g_ready[device]) return W4_OK;
  int prev = -1;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (prev != device && (e = cudaSetDevice(device)) != cudaSuccess)
    return cuda_fail(e, "cudaSetDevice");
  DeviceInfo di;
  int st = W4_OK;
  do {
    if ((e = cudaDeviceGetAttribute(&di.sm_count, cudaDevAttrMultiProcessorCount, device)) ||
        (e = cudaDeviceGetAttribute(&di.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin,
                                    device)) ||
        (e = cudaDeviceGetAttribute(&di.cc_major, cudaDevAttrComputeCapabilityMajor, device)) ||
        (e = cudaDeviceGetAttribute(&di.cc_minor, cudaDevAttrComputeCapabilityMinor, device))) {
      st = cuda_fail(e, "cudaDeviceGetAttribute");
      break;
    }
    if (di.cc_major != 10 || di.cc_minor != 0) {
      st = fail(W4_ERR_UNSUPPORTED,
                "device %d is sm_%d%d; this library is built for sm_100a (B200) only", device,
                di.cc_major, di.cc_minor);
      break;
    }
    if (!g_encode) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
      if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) {
        st = fail(W4_ERR_CUDA, "cannot resolve cuTensorMapEncodeTiled from the driver");
        break;
      }
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
    void* addr = nullptr;
    if ((e = cudaGetSymbolAddress(&addr, g_error_word)) != cudaSuccess) {
      st = cuda_fail(e, "cudaGetSymbolAddress(error word)");
      break;
    }
    di.err_word = static_cast<int*>(addr);
    st = gemv_init_device(di);
    if (st == W4_OK) st = decode_init_device(di);
    if (st == W4_OK) st = mega_init_device(di);
    if (st == W4_OK) st = gemm_init_device(di);
    if (st == W4_OK) st = gptq_init_device(di);
  } while (false);
  if (prev != device) cudaSetDevice(prev);
  if (st == W4_OK) {
    g_devices[device] = di;
    g_ready[device] = true;
  }
  return st;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_dtype(int dt, const char* what) {
  if (dt != W4_F16 && dt != W4_BF16)
    return fail(W4_ERR_INVALID_ARG, "%s dtype %d is neither W4_F16 nor W4_BF16", what, dt);
  return W4_OK;
}

}  // namespace
}  // namespace w4

using namespace w4;

extern "C" {

int w4_version(void) { return W4B200_VERSION; }

const char* w4_status_string(int status) {
  switch (status) {
    case W4_OK: return "W4_OK";
    case W4_ERR_INVALID_ARG: return "W4_ERR_INVALID_ARG";
    case W4_ERR_ALIGNMENT: return "W4_ERR_ALIGNMENT";
    case W4_ERR_UNSUPPORTED: return "W4_ERR_UNSUPPORTED";
    case W4_ERR_CUDA: return "W4_ERR_CUDA";
    case W4_ERR_DEVICE: return "W4_ERR_DEVICE";
    default: return "W4_ERR_UNKNOWN";
  }
}

const char* w4_last_error(void) { return g_last_error.c_str(); }

int w4_init(int device) {
  if (device < 0 || device >= kMaxDevices)
    return fail(W4_ERR_INVALID_ARG, "device %d out of range", device);
  std::lock_guard<std::mutex> lock(g_init_mutex);
  return init_locked(device);
}

int w4_pack(const void* w, int w_dtype, int32_t* packed, void* scales, int K, int N,
            int group_size, void* stream) {
  if (!w || !packed || !scales) return fail(W4_ERR_INVALID_ARG, "w4_pack: null pointer");
  if (w_dtype != W4_PACK_F16 && w_dtype != W4_PACK_BF16 && w_dtype != W4_PACK_F32)
    return fail(W4_ERR_INVALID_ARG, "w4_pack: w dtype %d unknown", w_dtype);
  if (K <= 0 || N <= 0) return fail(W4_ERR_INVALID_ARG, "w4_pack: K=%d N=%d", K, N);
  if (group_size <= 0 || group_size % 8 != 0 || K % group_size != 0)
    return fail(W4_ERR_INVALID_ARG,
                "w4_pack: group_size=%d must be a positive multiple of 8 dividing K=%d",
                group_size, K);
  int dev;
  int st = current_device(&dev);
  if (st != W4_OK) return st;
  cudaError_t e = launch_pack(w, w_dtype, packed, scales, K, N, group_size, (cudaStream_t)stream);
  return e == cudaSuccess ? W4_OK : cuda_fail(e, "w4_pack launch");
}

int w4_dequant(const int32_t* packed, const void* scales, void* out, int out_dtype, int K, int N,
               void* stream) {
  if (!packed || !scales || !out) return fail(W4_ERR_INVALID_ARG, "w4_dequant: null pointer");
  int st = check_dtype(out_dtype, "w4_dequant out");
  if (st != W4_OK) return st;
  if (K <= 0 || N <= 0 || K % 128 != 0 || N % 8 != 0)
    return fail(W4_ERR_INVALID_ARG, "w4_dequant: K=%d must be a multiple of 128, N=%d of 8", K,
                N);
  if (!aligned16(packed) || !aligned16(scales) || !aligned16(out))
    return fail(W4_ERR_ALIGNMENT, "w4_dequant: pointers must be 16-byte aligned");
  int dev;
  if ((st = current_device(&dev)) != W4_OK) return st;
  cudaError_t e = launch_dequant(packed, scales, out, out_dtype == W4_BF16, K, N,
                                 (cudaStream_t)stream);
  return e == cudaSuccess ? W4_OK : cuda_fail(e, "w4_dequant launch");
}

static int gemv_check(const void* x, int x_dtype, const int32_t* packed, const void* scales,
                      void* y, int y_dtype, int M, int K, int N) {
  if (!x || !packed || !scales || !y) return fail(W4_ERR_INVALID_ARG, "w4_gemv: null pointer");
  int st = check_dtype(x_dtype, "w4_gemv x");
  if (st != W4_OK) return st;
  if ((st = check_dtype(y_dtype, "w4_gemv y")) != W4_OK) return st;
  if (M < 1 || M > W4B200_MAX_M)
    return fail(W4_ERR_INVALID_ARG, "w4_gemv: M=%d outside 1..%d", M, W4B200_MAX_M);
  if (K <= 0 || K % 128 != 0)
    return fail(W4_ERR_INVALID_ARG, "w4_gemv: K=%d must be a positive multiple of 128", K);
  if (N <= 0 || N % 8 != 0)
    return fail(W4_ERR_INVALID_ARG, "w4_gemv: N=%d must be a positive multiple of 8", N);
  if (!aligned16(x) || !aligned16(packed) || !aligned16(scales) || !aligned16(y))
    return fail(W4_ERR_ALIGNMENT, "w4_gemv: pointers must be 16-byte aligned");
  return W4_OK;
}

int w4_gemv_tune(int M, int K, int N, int x_dtype, int y_dtype, int split_k, int num_warps,
                 w4_gemv_config* out, float* best_us) {
  if (!out) return fail(W4_ERR_INVALID_ARG, "w4_gemv_tune: null out");
  int st = check_dtype(x_dtype, "w4_gemv_tune x");
  if (st != W4_OK) return st;
  if ((st = check_dtype(y_dtype, "w4_gemv_tune y")) != W4_OK) return st;
  if (M < 1 || M > W4B200_MAX_M || K <= 0 || K % 128 != 0 || N <= 0 || N % 8 != 0)
    return fail(W4_ERR_INVALID_ARG, "w4_gemv_tune: M=%d K=%d N=%d", M, K, N);
  if (split_k > 16 || split_k > K / 128)
    return fail(W4_ERR_INVALID_ARG, "split_k=%d must be <= min(16, K/128=%d)", split_k, K / 128);
  if (num_warps > 0 && num_warps != 4 && num_warps != 8)
    return fail(W4_ERR_INVALID_ARG, "num_warps=%d must be 4 or 8", num_warps);
  return gemv_tune(M, K, N, x_dtype == W4_BF16, y_dtype == W4_BF16, split_k, num_warps, out,
                   best_us);
}

int w4_gemv_default_config(int M, int K, int N, int split_k, int num_warps,
                           w4_gemv_config* out) {
  if (!out) return fail(W4_ERR_INVALID_ARG, "w4_gemv_default_config: null out");
  if (M < 1 || M > W4B200_MAX_M || K <= 0 || K % 128 != 0 || N <= 0 || N % 8 != 0)
    return fail(W4_ERR_INVALID_ARG, "w4_gemv_default_config: M=%d K=%d N=%d", M, K, N);
  if (split_k > 16 || split_k > K / 128)
    return fail(W4_ERR_INVALID_ARG, "split_k=%d must be <= min(16, K/128=%d)", split_k, K / 128);
  if (num_warps > 0 && num_warps != 4 && num_warps != 8)
    return fail(W4_ERR_INVALID_ARG, "num_warps=%d must be 4 or 8", num_warps);
  int dev;
  int st = current_device(&dev);
  if (st != W4_OK) return st;
  return gemv_choose_config(M, K, N, split_k, num_warps, device_info(dev), out);
}

int w4_gemv(const void* x, int x_dtype, const int32_t* packed, const void* scales, void* y,
            int y_dtype, int M, int K, int N, int split_k, int num_warps, void* stream) {
  int st = gemv_check(x, x_dtype, packed, scales, y, y_dtype, M, K, N);
  if (st != W4_OK) return st;
  w4_gemv_config c;
  if ((st = w4_gemv_default_config(M, K, N, split_k, num_warps, &c)) != W4_OK) return st;
  GemvLaunch L{x, packed, scales, y, x_dtype == W4_BF16, y_dtype == W4_BF16, M, K, N, c, {}};
  return launch_gemv(L, (cudaStream_t)stream);
}

int w4_gemv_ex(const void* x, int x_dtype, const int32_t* packed, const void* scales, void* y,
               int y_dtype, int M, int K, int N, const w4_gemv_config* cfg, void* stream) {
  int st = gemv_check(x, x_dtype, packed, scales, y, y_dtype, M, K, N);
  if (st != W4_OK) return st;
  if (!cfg) return fail(W4_ERR_INVALID_ARG, "w4_gemv_ex: null config");
  GemvLaunch L{x, packed, scales, y, x_dtype == W4_BF16, y_dtype == W4_BF16, M, K, N, *cfg, {}};
  return launch_gemv(L, (cudaStream_t)stream);
}

int w4_gemv_plan_create(const int32_t* packed, const void* scales, int M, int K, int N,
                        int x_dtype, int y_dtype, const w4_gemv_config* cfg,
                        w4_gemv_plan** plan) {
  if (!plan) return fail(W4_ERR_INVALID_ARG, "w4_gemv_plan_create: null plan");
  *plan = nullptr;
  // x and y are bound at launch: check the rest with stand-in aligned pointers
  static const int16_t stand_in[8] __attribute__((aligned(16))) = {};
  int st = gemv_check(stand_in, x_dtype, packed, scales, (void*)stand_in, y_dtype, M, K, N);
  if (st != W4_OK) return st;
  w4_gemv_config c;
  if (cfg) {
    c = *cfg;
  } else if ((st = w4_gemv_default_config(M, K, N, 0, 0, &c)) != W4_OK) {
    return st;
  }
  GemvLaunch L{nullptr, packed, scales, nullptr, x_dtype == W4_BF16, y_dtype == W4_BF16,
               M, K, N, c, {}};
  void* h = nullptr;
  if ((st = gemv_plan_create(L, &h)) != W4_OK) return st;
  *plan = static_cast<w4_gemv_plan*>(h);
  return W4_OK;
}

int w4_gemv_plan_launch(const w4_gemv_plan* plan, const void* x, void* y, void* stream) {
  return w4_gemv_plan_launch_host(plan, nullptr, const_cast<void*>(x), y, nullptr, stream);
}

int w4_gemv_plan_launch_host(const w4_gemv_plan* plan, const void* x_host, void* x, void* y,
                             void* y_host, void* stream) {
  if (!plan || !x || !y) return fail(W4_ERR_INVALID_ARG, "w4_gemv_plan_launch: null argument");
  if (!aligned16(x) || !aligned16(y))
    return fail(W4_ERR_ALIGNMENT, "w4_gemv_plan_launch: x and y must be 16-byte aligned");
  return gemv_plan_launch(plan, x_host, x, y, y_host, (cudaStream_t)stream);
}

int w4_gemv_plans_launch_host(const w4_gemv_plan* const* plans, int n, const void* x_host,
                              void* x, void* y, void* y_host, void* stream) {
  if (!plans || n < 1 || !x || !y)
    return fail(W4_ERR_INVALID_ARG, "w4_gemv_plans_launch_host: null argument or n < 1");
  for (int i = 0; i < n; ++i)
    if (!plans[i]) return fail(W4_ERR_INVALID_ARG, "w4_gemv_plans_launch_host: plan %d null", i);
  if (!aligned16(x) || !aligned16(y))
    return fail(W4_ERR_ALIGNMENT, "w4_gemv_plans_launch_host: x and y must be 16-byte aligned");
  return gemv_plans_launch(reinterpret_cast<const void* const*>(plans), n, x_host, x, y, y_host,
                           (cudaStream_t)stream);
}

int w4_gemv_plan_destroy(w4_gemv_plan* plan) {
  gemv_plan_destroy(plan);
  return W4_OK;
}

int w4_gemv_fused(const void* x, int x_dtype, const int32_t* packed, const void* scales,
                  void* y, int y_dtype, int M, int K, int N, const w4_fused_ops* ops,
                  const w4_gemv_config* cfg, void* stream) {
  int st = gemv_check(x, x_dtype, packed, scales, y, y_dtype, M, K, N);
  if (st != W4_OK) return st;
  if (!cfg || !ops) return fail(W4_ERR_INVALID_ARG, "w4_gemv_fused: null config or ops");
  if (ops->prologue < W4_PRO_NONE || ops->prologue > W4_PRO_SWIGLU)
    return fail(W4_ERR_INVALID_ARG, "w4_gemv_fused: prologue %d unknown", ops->prologue);
  if (ops->epilogue < W4_EPI_NONE || ops->epilogue > W4_EPI_SWIGLU)
    return fail(W4_ERR_INVALID_ARG, "w4_gemv_fused: epilogue %d unknown", ops->epilogue);
  if (ops->epilogue == W4_EPI_SWIGLU &&
      (cfg->split != 1 || cfg->strips < 1 || N % (32 * cfg->strips) != 0 || x_dtype != W4_BF16 ||
       M > 8))
    return fail(W4_ERR_UNSUPPORTED,
                "w4_gemv_fused: the SwiGLU epilogue needs split = 1, N a multiple of the tile "
                "(32 * strips), bf16 x and at most 8 rows");
  if (ops->prologue == W4_PRO_RMSNORM && (!ops->norm_weight || !aligned16(ops->norm_weight)))
    return fail(W4_ERR_ALIGNMENT, "w4_gemv_fused: RMSNorm weight missing or not 16-byte aligned");
  if (ops->prologue != W4_PRO_NONE && x_dtype != y_dtype)
    return fail(W4_ERR_INVALID_ARG, "w4_gemv_fused: a prologue needs x and y of one type");
  if ((ops->epilogue == W4_EPI_BIAS || ops->epilogue == W4_EPI_RESIDUAL) && !ops->epi_src)
    return fail(W4_ERR_INVALID_ARG, "w4_gemv_fused: epilogue source missing");
  GemvLaunch L{x, packed, scales, y, x_dtype == W4_BF16, y_dtype == W4_BF16, M, K, N, *cfg,
               *ops};
  return launch_gemv(L, (cudaStream_t)stream);
}

int w4_gemm(const void* x, int x_dtype, const int32_t* packed, const void* scales, void* y,
            int y_dtype, int M, int K, int N, void* stream) {
  return w4_gemm_ex(x, x_dtype, packed, scales, y, y_dtype, M, K, N, 0, stream);
}

int w4_gemm_ex(const void* x, int x_dtype, const int32_t* packed, const void* scales, void* y,
               int y_dtype, int M, int K, int N, int split_k, void* stream) {
  if (!x || !packed || !scales || !y) return fail(W4_ERR_INVALID_ARG, "w4_gemm: null pointer");
  if (split_k < 0 || split_k > 8 || (split_k > 0 && split_k > K / 64))
    return fail(W4_ERR_INVALID_ARG, "w4_gemm: split_k=%d (0 = choose, else 1..8 and <= K/64)",
                split_k);
  int st = check_dtype(x_dtype, "w4_gemm x");
  if (st != W4_OK) return st;
  if ((st = check_dtype(y_dtype, "w4_gemm y")) != W4_OK) return st;
  if (M < 1 || K <= 0 || K % 128 != 0 || N <= 0 || N % 128 != 0)
    return fail(W4_ERR_INVALID_ARG,
                "w4_gemm: M=%d K=%d N=%d (M >= 1, K and N multiples of 128)", M, K, N);
  if (!aligned16(x) || !aligned16(packed) || !aligned16(scales) || !aligned16(y))
    return fail(W4_ERR_ALIGNMENT, "w4_gemm: pointers must be 16-byte aligned");
  return launch_gemm(x, x_dtype == W4_BF16, packed, scales, y, y_dtype == W4_BF16, M, K, N,
                     split_k, (cudaStream_t)stream);
}

int w4_gptq_block(const float* w, const float* hinv, int N, int32_t* packed, void* scales,
                  float* err, void* stream) {
  if (!w || !hinv || !packed || !scales || !err)
    return fail(W4_ERR_INVALID_ARG, "w4_gptq_block: null pointer");
  if (N <= 0) return fail(W4_ERR_INVALID_ARG, "w4_gptq_block: N=%d", N);
  const uintptr_t a = reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(hinv) |
                      reinterpret_cast<uintptr_t>(packed) | reinterpret_cast<uintptr_t>(err);
  if ((a & 3u) != 0 || (reinterpret_cast<uintptr_t>(scales) & 1u) != 0)
    return fail(W4_ERR_ALIGNMENT, "w4_gptq_block: misaligned pointer");
  int dev = 0;
  const int st = current_device(&dev);  // initialises the device on first use
  if (st != W4_OK) return st;
  return launch_gptq_block(w, hinv, N, packed, scales, err, (cudaStream_t)stream);
}

size_t w4_peer_flag_bytes(int world) {
  (void)world;
  return 256;  // flag words at 0 (one per rank, <= 8), state words at 128
}

int w4_gemv_allgather(const void* x, int x_dtype, const int32_t* packed, const void* scales,
                      int y_dtype, int M, int K, int N, const w4_gemv_config* cfg,
                      const w4_peer_out* peers, void* stream) {
  if (!cfg || !peers) return fail(W4_ERR_INVALID_ARG, "w4_gemv_allgather: null config or peers");
  const w4_peer_out& po = *peers;
  if (po.world < 1 || po.world > W4B200_MAX_PEERS || po.rank < 0 || po.rank >= po.world)
    return fail(W4_ERR_INVALID_ARG, "w4_gemv_allgather: rank %d of %d (at most %d ranks)",
                po.rank, po.world, W4B200_MAX_PEERS);
  if (po.col_off < 0 || po.n_full < po.col_off + N || po.col_off % 8 != 0 || po.n_full % 8 != 0)
    return fail(W4_ERR_INVALID_ARG,
                "w4_gemv_allgather: columns [%d, %d) outside n_full=%d (multiples of 8)",
                po.col_off, po.col_off + N, po.n_full);
  if (!po.state || (reinterpret_cast<uintptr_t>(po.state) & 3))
    return fail(W4_ERR_INVALID_ARG, "w4_gemv_allgather: state words missing");
  for (int q = 0; q < po.world; ++q) {
    if (!po.flags[q] || !po.y[0][q] || !po.y[1][q])
      return fail(W4_ERR_INVALID_ARG, "w4_gemv_allgather: buffers of rank %d missing", q);
    if (!aligned16(po.y[0][q]) || !aligned16(po.y[1][q]))
      return fail(W4_ERR_ALIGNMENT, "w4_gemv_allgather: y buffers must be 16-byte aligned");
  }
  // the local y argument of the plain check: this rank's own buffer
  int st = gemv_check(x, x_dtype, packed, scales, po.y[0][po.rank], y_dtype, M, K, N);
  if (st != W4_OK) return st;
  w4_fused_ops ops{};
  GemvLaunch L{x, packed, scales, po.y[0][po.rank], x_dtype == W4_BF16, y_dtype == W4_BF16,
               M, K, N, *cfg, ops, &po};
  return launch_gemv(L, (cudaStream_t)stream);
}

static_assert(sizeof(cudaIpcMemHandle_t) == W4B200_IPC_HANDLE_BYTES, "IPC handle size");

int w4_peer_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return fail(W4_ERR_INVALID_ARG, "w4_peer_alloc: arguments");
  int dev;
  int st = current_device(&dev);
  if (st != W4_OK) return st;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "w4_peer_alloc cudaMalloc");
  // The zeroing must have landed before any peer can map the buffer: a peer's
  // first flag store could otherwise be wiped by a memset still in flight.
  if ((e = cudaMemset(*ptr, 0, bytes)) != cudaSuccess ||
      (e = cudaDeviceSynchronize()) != cudaSuccess ||
      (e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), *ptr)) != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return cuda_fail(e, "w4_peer_alloc");
  }
  return W4_OK;
}

int w4_peer_free(void* ptr) {
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? W4_OK : cuda_fail(e, "w4_peer_free");
}

int w4_peer_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return fail(W4_ERR_INVALID_ARG, "w4_peer_open: arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? W4_OK : cuda_fail(e, "w4_peer_open");
}

int w4_peer_close(void* ptr) {
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? W4_OK : cuda_fail(e, "w4_peer_close");
}

int w4_decode_embed(const void* embed, int vocab, int hidden, const int64_t* prompt,
                    const int64_t* prompt_len, int64_t* token, const int64_t* pos, void* h,
                    int pdl, void* stream) {
  if (!embed || !prompt || !prompt_len || !token || !pos || !h)
    return fail(W4_ERR_INVALID_ARG, "w4_decode_embed: null pointer");
  if (vocab <= 0 || hidden <= 0 || hidden % 8 != 0)
    return fail(W4_ERR_INVALID_ARG, "w4_decode_embed: vocab=%d hidden=%d", vocab, hidden);
  if (!aligned16(embed) || !aligned16(h))
    return fail(W4_ERR_ALIGNMENT, "w4_decode_embed: embed/h must be 16-byte aligned");
  int dev;
  int st = current_device(&dev);
  if (st != W4_OK) return st;
  return launch_decode_embed(embed, vocab, hidden, prompt, prompt_len, token, pos, h, pdl,
                             (cudaStream_t)stream);
}

int w4_decode_attention(const void* qkv, const void* cos_table, const void* sin_table,
                        const int64_t* pos, void* k_cache, void* v_cache, void* out, int heads,
                        int kv_heads, int head_dim, int max_seq, int pdl, void* stream) {
  if (!qkv || !cos_table || !sin_table || !pos || !k_cache || !v_cache || !out)
    return fail(W4_ERR_INVALID_ARG, "w4_decode_attention: null pointer");
  if (head_dim != 128)
    return fail(W4_ERR_UNSUPPORTED, "w4_decode_attention: head_dim %d (128 only)", head_dim);
  if (kv_heads <= 0 || heads <= 0 || heads % kv_heads != 0 || heads / kv_heads > 16)
    return fail(W4_ERR_INVALID_ARG, "w4_decode_attention: heads=%d kv_heads=%d", heads, kv_heads);
  if (max_seq <= 0 || max_seq > 16384)
    return fail(W4_ERR_INVALID_ARG, "w4_decode_attention: max_seq=%d outside 1..16384", max_seq);
  int dev;
  int st = current_device(&dev);
  if (st != W4_OK) return st;
  return launch_decode_attention(qkv, cos_table, sin_table, pos, k_cache, v_cache, out, heads,
                                 kv_heads, max_seq, pdl, (cudaStream_t)stream);
}

size_t w4_lm_head_workspace_bytes(void) { return lm_head_workspace_bytes(); }

int w4_lm_head_argmax(const void* h, const void* norm_weight, float eps, const void* embed,
                      int vocab, int hidden, void* logits, int64_t* token, int64_t* pos,
                      void* workspace, size_t workspace_bytes, int pdl, void* stream) {
  if (!h || !norm_weight || !embed || !token || !pos || !workspace)
    return fail(W4_ERR_INVALID_ARG, "w4_lm_head_argmax: null pointer");
  if (workspace_bytes < lm_head_workspace_bytes())
    return fail(W4_ERR_INVALID_ARG, "w4_lm_head_argmax: workspace of %zu bytes < %zu",
                workspace_bytes, lm_head_workspace_bytes());
  if (vocab <= 0) return fail(W4_ERR_INVALID_ARG, "w4_lm_head_argmax: vocab=%d", vocab);
  if (!lm_head_hidden_supported(hidden))
    return fail(W4_ERR_UNSUPPORTED,
                "w4_lm_head_argmax: hidden=%d not in {256, 512, 1024, 1536, 2048}", hidden);
  if (!aligned16(h) || !aligned16(norm_weight) || !aligned16(embed) ||
      (logits && !aligned16(logits)) || !aligned16(workspace))
    return fail(W4_ERR_ALIGNMENT, "w4_lm_head_argmax: pointers must be 16-byte aligned");
  int dev;
  int st = current_device(&dev);
  if (st != W4_OK) return st;
  return launch_lm_head_argmax(h, norm_weight, eps, embed, vocab, hidden, logits, token, pos,
                               workspace, pdl, (cudaStream_t)stream);
}

int w4_lm_head_argmax_static(const void* h, const void* norm_weight, float eps,
                             const void* embed, int vocab, int hidden, void* logits,
                             int64_t* token, int64_t* pos, int pdl, void* stream) {
  if (!h || !norm_weight || !embed || !token || !pos)
    return fail(W4_ERR_INVALID_ARG, "w4_lm_head_argmax_static: null pointer");
  // the state in the static array is the same few words whatever the vocab:
  // any positive int vocab fits its 32-bit row index
  if (vocab <= 0) return fail(W4_ERR_INVALID_ARG, "w4_lm_head_argmax_static: vocab=%d", vocab);
  // checked before the first call's look-up and clearing of the array
  if (!lm_head_hidden_supported(hidden))
    return fail(W4_ERR_UNSUPPORTED,
                "w4_lm_head_argmax_static: hidden=%d not in {256, 512, 1024, 1536, 2048}",
                hidden);
  if (!aligned16(h) || !aligned16(norm_weight) || !aligned16(embed) ||
      (logits && !aligned16(logits)))
    return fail(W4_ERR_ALIGNMENT, "w4_lm_head_argmax_static: pointers must be 16-byte aligned");
  int dev;
  int st = current_device(&dev);
  if (st != W4_OK) return st;
  return lm_head_argmax_static(h, norm_weight, eps, embed, vocab, hidden, logits, token, pos,
                               pdl, (cudaStream_t)stream);
}

int w4_decode_step_scratch_bytes(const w4_decode_model* model, size_t* bytes) {
  if (!model || !bytes) return fail(W4_ERR_INVALID_ARG, "w4_decode_step_scratch_bytes: null");
  return decode_step_scratch_bytes(*model, bytes);
}

int w4_decode_step(const w4_decode_model* model, void* scratch, size_t scratch_bytes,
                   void* stream) {
  if (!model) return fail(W4_ERR_INVALID_ARG, "w4_decode_step: null model");
  return launch_decode_step(*model, scratch, scratch_bytes, (cudaStream_t)stream);
}

int w4_device_error(int device, int* code) {
  if (!code) return fail(W4_ERR_INVALID_ARG, "w4_device_error: null out");
  int st = w4_init(device);
  if (st != W4_OK) return st;
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != device) cudaSetDevice(device);
  int zero = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(code, g_error_word, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_error_word, &zero, sizeof(int));
  if (prev != device) cudaSetDevice(prev);
  return e == cudaSuccess ? W4_OK : cuda_fail(e, "w4_device_error");
}

}  // extern "C"
