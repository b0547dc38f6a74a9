/*
 * w4b200.h - C ABI of the B200 (sm_100a) W4A16 dequantise + GEMV library.
 *
 * Weight format (the reference's, kept bit for bit):
 *   packed : int32 [K/8, N], row-major (N contiguous). Word (j, n) holds the
 *            8 nibbles of W[8j .. 8j+7, n]; nibble i sits at bits 4i..4i+3 and
 *            stores q = clamp(round_half_even(w / s) + 8, 0, 15).
 *   scales : fp16 [K/group, N], row-major, s = fp16(max|w| / 7) per (group, n).
 *   dequant: w = (q - 8) * s.
 * Activations x are [M, K] row-major fp16 or bf16 (M = 1 is batch-1 decode),
 * outputs y are [M, N] row-major fp16 or bf16.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * passed as void*. None of them allocates, frees or synchronises, so they
 * can be recorded into a CUDA graph once w4_init() has run on the device.
 * All return a w4_status; a non-zero status means nothing was launched.
 */
#ifndef W4B200_H_
#define W4B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define W4B200_VERSION 100 /* 1.0.0 */
#define W4B200_GROUP_SIZE 128
#define W4B200_MAX_M 16

typedef enum {
  W4_OK = 0,
  W4_ERR_INVALID_ARG = 1, /* bad sizes, null pointers, unknown dtype   */
  W4_ERR_ALIGNMENT = 2,   /* pointer or row pitch not 16-byte aligned  */
  W4_ERR_UNSUPPORTED = 3, /* valid request this build does not cover   */
  W4_ERR_CUDA = 4,        /* a CUDA runtime call failed (see message)  */
  W4_ERR_DEVICE = 5       /* a kernel reported a timed-out wait        */
} w4_status;

typedef enum { W4_F16 = 0, W4_BF16 = 1 } w4_dtype;

/* Tile configuration of the fused GEMV. Zero fields mean "choose". */
typedef struct {
  int strips;     /* 32-column strips per CTA: 1, 2 or 4 (tile = 32*strips)  */
  int row_groups; /* 128-row K groups per pipeline stage and strip: 1,2,4,8  */
  int stages;     /* shared-memory pipeline depth, 2..8                      */
  int split;      /* CTAs per cluster along K (deterministic DSMEM reduce)   */
  int pdl;        /* 1: launch with programmatic dependent launch            */
} w4_gemv_config;

/* Library version (W4B200_VERSION). */
int w4_version(void);

/* Human-readable name of a status code. */
const char* w4_status_string(int status);

/* Message of the last failure on the calling host thread ("" if none). */
const char* w4_last_error(void);

/* One-off per-device set-up: resolves the driver's tensor-map encoder and
 * raises the kernels' shared-memory limits. Called implicitly by every entry
 * point; call it explicitly before capturing a CUDA graph. */
int w4_init(int device);

/* Input element types accepted by w4_pack (the reference packer quantises
 * w.float(), whatever the float type of w). */
typedef enum { W4_PACK_F16 = 0, W4_PACK_BF16 = 1, W4_PACK_F32 = 2 } w4_pack_dtype;

/* Replaces roofline/kernels.py:24-47 pack_weights (the reference runs it as
 * torch ops on whatever device holds w). w: [K, N] row-major device pointer
 * of type w_dtype. Writes packed int32 [K/8, N] and fp16 scales
 * [K/group_size, N]. Bit-exact with the reference for every group whose
 * scale is non-zero; where w/s is NaN (an all-zero group, whose fp16 scale
 * underflows to 0) it stores nibble 0, the value torch's NaN-to-int32 cast
 * gives on a CUDA device. */
int w4_pack(const void* w, int w_dtype, int32_t* packed, void* scales, int K,
            int N, int group_size, void* stream);

/* Replaces roofline/kernels.py:77-90 dequantize_v1 (_dequant_kernel,
 * kernels.py:50-74): out[k, n] = round((q - 8) * s) to out_dtype, the
 * product taken in fp32. Bit-exact with the reference for fp16 output. */
int w4_dequant(const int32_t* packed, const void* scales, void* out,
               int out_dtype, int K, int N, void* stream);

/* Replaces roofline/kernels.py:131-145 gemv_v2 (M = 1) and
 * roofline/kernels.py:250-268 gemv_v3 (split_k, num_warps): fused
 * y[m, n] = sum_k x[m, k] * (q[k, n] - 8) * s[k / 128, n], fp32 accumulation
 * on the tensor cores, one rounding to y_dtype at the end.
 *   split_k   <= 0 picks the split; otherwise K is cut into split_k slices
 *             reduced in a fixed order (no atomics: results do not depend on
 *             scheduling). split_k must be <= 16.
 *   num_warps <= 0 picks the tile; 4 or 8 asks for that many compute warps.
 * Requirements: 1 <= M <= 16, K % 128 == 0, N % 8 == 0, all pointers 16-byte
 * aligned. packed/scales must not be written by the kernel launched just
 * before on the same stream when pdl is on (their loads start before the
 * grid-dependency wait; x is read only after it). */
int w4_gemv(const void* x, int x_dtype, const int32_t* packed,
            const void* scales, void* y, int y_dtype, int M, int K, int N,
            int split_k, int num_warps, void* stream);

/* Same as w4_gemv with an explicit tile configuration (used by the tuner). */
int w4_gemv_ex(const void* x, int x_dtype, const int32_t* packed,
               const void* scales, void* y, int y_dtype, int M, int K, int N,
               const w4_gemv_config* cfg, void* stream);

/* The configuration w4_gemv would use for (M, K, N, split_k, num_warps).
 * Replaces the choice made by roofline/kernels.py:211-247 _tune_num_warps
 * when no tuned entry exists. */
int w4_gemv_default_config(int M, int K, int N, int split_k, int num_warps,
                           w4_gemv_config* out);

/* Reads and clears the device-side error word that kernels set when a
 * bounded wait gives up (0 = no error). Synchronises the device. */
int w4_device_error(int device, int* code);

#ifdef __cplusplus
}
#endif

#endif /* W4B200_H_ */
