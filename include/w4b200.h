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
 * passed as void*. None of the compute entry points allocates, frees or
 * synchronises, so they can be recorded into a CUDA graph once w4_init()
 * has run on the device. The exceptions, which belong outside any capture:
 * w4_gemv_tune (a set-up call that allocates and synchronises) and the
 * w4_peer_* memory calls near the end (they allocate, map and free).
 * All return a w4_status; a non-zero status means nothing was launched.
 */
#ifndef W4B200_H_
#define W4B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define W4B200_VERSION 110 /* 1.1.0 */
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
  int columns;    /* CTA columns along N: 0 = one CTA per column tile; C less
                   * than the tile count T gives CTA column i the tiles
                   * i, i + C, i + 2C, ..., streamed back to back (a GPU-
                   * filling grid for large N; 16 compute warps, strips x
                   * row_groups = 2 x 8 or 4 x 4, exist in this mode only).
                   * C < T needs no epilogue and a local output
                   * (W4_ERR_UNSUPPORTED otherwise).                         */
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

/* A GEMV launch prepared once and replayed: tile, kernel instance, encoded
 * tensor maps and launch geometry for fixed weights, shape and dtypes.
 * Replaces the per-call work of roofline/kernels.py:250-268 gemv_v3 (tune-
 * cache lookup, argument set-up, launch) for a loop that calls the same
 * layer many times: a launch through a plan only binds x, y and the stream.
 * cfg may be NULL (the w4_gemv_default_config tile). Creating a plan
 * allocates host memory only; destroy it with w4_gemv_plan_destroy. A plan
 * belongs to the device that was current when it was made. */
typedef struct w4_gemv_plan w4_gemv_plan;
int w4_gemv_plan_create(const int32_t* packed, const void* scales, int M, int K,
                        int N, int x_dtype, int y_dtype,
                        const w4_gemv_config* cfg, w4_gemv_plan** plan);
/* y = x @ dequant(W) with the plan's tile (x, y 16-byte aligned device
 * pointers of the plan's dtypes). */
int w4_gemv_plan_launch(const w4_gemv_plan* plan, const void* x, void* y,
                        void* stream);
/* The same with host buffers: x_host (M*K elements) is copied into x before
 * the GEMV and y into y_host (M*N elements) after it, all enqueued on
 * `stream` (pinned host memory makes the copies asynchronous). x_host or
 * y_host may be NULL to skip that copy. */
int w4_gemv_plan_launch_host(const w4_gemv_plan* plan, const void* x_host,
                             void* x, void* y, void* y_host, void* stream);
/* Several plans in one call, with host buffers (a decode step's GEMVs that
 * take their inputs from the host, say). The inputs of every plan lie back to
 * back in x_host (plan i's M*K elements after plan i-1's) and are copied into
 * x with one copy; the GEMVs run in order, plan i reading its slice of x and
 * writing its slice of y (its M*N elements, back to back); y is copied into
 * y_host with one copy. x_host or y_host may be NULL to skip that copy. */
int w4_gemv_plans_launch_host(const w4_gemv_plan* const* plans, int n,
                              const void* x_host, void* x, void* y, void* y_host,
                              void* stream);
int w4_gemv_plan_destroy(w4_gemv_plan* plan);

/* The configuration w4_gemv would use for (M, K, N, split_k, num_warps).
 * Replaces the choice made by roofline/kernels.py:211-247 _tune_num_warps
 * when no tuned entry exists. */
int w4_gemv_default_config(int M, int K, int N, int split_k, int num_warps,
                           w4_gemv_config* out);

/* Replaces roofline/kernels.py:211-247 _tune_num_warps for hosts outside
 * Python: times the fused GEMV's tile candidates for (M, K, N) on the current
 * device and writes the fastest to *out (pdl = 0) and, if best_us is not
 * NULL, its time per launch. Each candidate runs as one CUDA graph of
 * dependent launches, each on its own copy of random weights, the copies
 * together exceeding 3x L2, so the time is that of a GEMV in a decode chain
 * (a lone microsecond launch cannot be timed). split_k / num_warps <= 0 leave
 * the split / the compute warps free; otherwise they are fixed, as in
 * w4_gemv. A set-up call: it allocates and frees device memory (up to a few
 * GB for the largest shapes) and synchronises, so it must not run during
 * stream capture. */
int w4_gemv_tune(int M, int K, int N, int x_dtype, int y_dtype, int split_k,
                 int num_warps, w4_gemv_config* out, float* best_us);

/* Operations fused into the GEMV for a decode step. */
typedef enum { W4_PRO_NONE = 0, W4_PRO_RMSNORM = 1, W4_PRO_SWIGLU = 2 } w4_prologue;
typedef enum {
  W4_EPI_NONE = 0,
  W4_EPI_BIAS = 1,
  W4_EPI_RESIDUAL = 2,
  W4_EPI_SWIGLU = 3
} w4_epilogue;
typedef struct {
  int prologue;            /* W4_PRO_RMSNORM: x <- rmsnorm(x) * norm_weight;
                              W4_PRO_SWIGLU : x is [M, 2K] gate|up, x <- silu(gate) * up */
  const void* norm_weight; /* RMSNorm weight [K] (x's type), 16-byte aligned */
  float eps;               /* RMSNorm epsilon */
  int epilogue;            /* W4_EPI_BIAS: y <- y + bias[n];
                              W4_EPI_RESIDUAL: y <- residual + round(y) (may alias y);
                              W4_EPI_SWIGLU: the columns hold gate and up in alternating
                              blocks of B = 16 * strips (gate 0..B-1, up 0..B-1, gate
                              B..2B-1, ...), and y [M, N/2] <-
                              round(round(silu(round(gate))) * round(up)). Needs split = 1
                              and bf16 x with at most 8 rows; epi_src unused */
  const void* epi_src;     /* bias [N] or residual [M, N] (y's type) */
} w4_fused_ops;

/* w4_gemv_ex with fused prologue/epilogue (the decoder layer's RMSNorm,
 * SwiGLU, q/k/v bias and residual adds of scripts/decode_loop.py's HF
 * forward, which ran them as separate torch ops around W4Linear). */
int w4_gemv_fused(const void* x, int x_dtype, const int32_t* packed,
                  const void* scales, void* y, int y_dtype, int M, int K, int N,
                  const w4_fused_ops* ops, const w4_gemv_config* cfg,
                  void* stream);

/* w4_gemm: y[M, N] = x[M, K] @ dequantize_v1(packed, scales) on the
 * tensor cores (tcgen05, fp32 accumulate) for any M - the prefill rows of
 * W4Linear, which the reference runs as dequantize_v1 (kernels.py:77-90)
 * into an fp16 [K, N] copy followed by an fp32 matmul
 * (scripts/decode_loop.py:51-55). The dequantised tile stays in shared
 * memory. fp16 x uses the reference's fp16 weights fp16((q - 8) * s); bf16 x
 * uses bf16((q - 8) * s). K and N multiples of 128, pointers 16-byte
 * aligned. */
int w4_gemm(const void* x, int x_dtype, const int32_t* packed, const void* scales,
            void* y, int y_dtype, int M, int K, int N, void* stream);
/* Same, with the K split fixed: split_k = 0 lets the library choose (grids of
 * fewer tiles than SMs cut K into slices; a last wave of a few tiles goes to a
 * second, programmatically dependent launch of K-sliced tiles), 1..8 runs one
 * launch of 128-column tiles with K cut into that many slices (<= K/64).
 * The slices of a tile form a cluster and are summed over DSMEM in rank
 * order: results do not depend on scheduling. */
int w4_gemm_ex(const void* x, int x_dtype, const int32_t* packed, const void* scales,
               void* y, int y_dtype, int M, int K, int N, int split_k, void* stream);

/* Calibrated int4 packing (GPTQ), the step the reference lists after its
 * round-to-nearest packer (devto_article.md:71), in the same packed format
 * (kernels.py:24-47). One call quantises one 128-row block of W [K, N]
 * (K = in-features; the block is one scale group):
 *   w      fp32 [128, N], the block's rows after the error feedback of the
 *          earlier blocks (read only);
 *   hinv   fp32 [128, 128] row-major, the block's diagonal block of U, the
 *          upper Cholesky factor of the conditioned inverse Hessian
 *          (H^-1 = U^T U, H = X^T X over calibration inputs);
 *   packed int32 [16, N], the block's 16 packed rows;
 *   scales fp16 [N], the block's scale row: fp16(max|w| / 7) over the
 *          error-compensated rows, as the reference packer computes it;
 *   err    fp32 [128, N], (w_i - dequant(q_i)) / U_ii per row, for the host's
 *          update of the later rows: W[b1:] -= U[b0:b1, b1:]^T @ err.
 * Rows are quantised in order; each row's error is fed back into the later
 * rows of the block. With U diagonal the result is the reference packer's. */
int w4_gptq_block(const float* w, const float* hinv, int N, int32_t* packed,
                  void* scales, float* err, void* stream);

/* ---------------------------------------------------------------------
 * Column-parallel GEMV with the all-gather fused into its epilogue.
 *
 * The reference runs on one GPU; its GEMV entry points
 * (src/roofline/kernels.py:131-145, :250-268) are sharded here over the
 * ranks of one node, column-parallel on N, as an NCCL all-gather after a
 * local GEMV would be. Instead of that collective, every rank's kernel
 * stores its slice of y straight into every rank's output buffer over
 * NVLink (plain peer stores), and the last CTA of each rank publishes an
 * epoch flag to every peer and waits (bounded) for all peers' flags. When
 * the kernel completes, y is whole on every rank.
 *
 * Buffers come from w4_peer_alloc on each rank and are opened on the others
 * with w4_peer_open (CUDA IPC). The output alternates between two buffers by
 * epoch parity, so a rank that runs ahead never overwrites a y that a slower
 * rank may still read; the k-th call on a group (counting from 1) writes
 * y[k % 2]. */
#define W4B200_MAX_PEERS 8
typedef struct w4_peer_out {
  int world, rank;             /* ranks in the group, this rank */
  int n_full;                  /* columns of the whole y */
  int col_off;                 /* first column of this rank's slice */
  void* y[2][W4B200_MAX_PEERS];          /* rank q's y buffers [M, n_full] by parity */
  unsigned* flags[W4B200_MAX_PEERS];     /* rank q's flag words (world of them) */
  unsigned* state;             /* this rank's own state words (zeroed once): epoch, done */
} w4_peer_out;

/* Bytes of the flag and state words a rank allocates for a group of `world`
 * ranks (one region: flags first, then the state). */
size_t w4_peer_flag_bytes(int world);

/* y = x @ dequant(W_local) on this rank's columns, gathered into every
 * rank's y[epoch % 2] (see above). N is the local column count; y_dtype the
 * type of y. Blocks (bounded, 1 s) until every rank of the group ran the same
 * call; a rank that never arrives sets the device error word. The epoch
 * counter lives on the device (state[0]); the host counts its own calls on
 * the group to know which of y[0] / y[1] the k-th call filled (y[k % 2],
 * k counted from 1). */
int w4_gemv_allgather(const void* x, int x_dtype, const int32_t* packed,
                      const void* scales, int y_dtype, int M, int K, int N,
                      const w4_gemv_config* cfg, const w4_peer_out* peers,
                      void* stream);

/* Device memory another process on this node can map: cudaMalloc plus its
 * IPC handle (W4B200_IPC_HANDLE_BYTES bytes written to handle). The memory is
 * zeroed, and the zeroing has completed on the device, before the handle is
 * returned (the call synchronises the device). */
#define W4B200_IPC_HANDLE_BYTES 64
int w4_peer_alloc(size_t bytes, void** ptr, void* handle);
int w4_peer_free(void* ptr);
/* Maps a peer's allocation into this process (peer access enabled). */
int w4_peer_open(const void* handle, void** ptr);
int w4_peer_close(void* ptr);

/* Decode-step kernels (bf16 activations), the rest of the batch-1 greedy
 * step that scripts/decode_loop.py:106-124 ran as an HF forward. All read
 * the step state (token, position) from device memory, so a whole step can
 * be captured once in a CUDA graph; pdl != 0 launches them with
 * programmatic dependent launch.
 *
 * w4_decode_embed: token <- pos < prompt_len ? prompt[pos] : token;
 *   h[hidden] <- embed[token, :]. */
int w4_decode_embed(const void* embed, int vocab, int hidden,
                    const int64_t* prompt, const int64_t* prompt_len,
                    int64_t* token, const int64_t* pos, void* h, int pdl,
                    void* stream);

/* w4_decode_attention: RoPE (rotate-half; cos/sin tables [max_seq,
 * head_dim]) on q and k of qkv = [q (heads*hd) | k (kv*hd) | v (kv*hd)],
 * k and v stored at position pos of the layer's caches [kv, max_seq, hd],
 * then GQA attention of every q head over positions 0..pos with softmax in
 * fp32; out [heads*hd]. head_dim must be 128. */
int w4_decode_attention(const void* qkv, const void* cos_table,
                        const void* sin_table, const int64_t* pos,
                        void* k_cache, void* v_cache, void* out, int heads,
                        int kv_heads, int head_dim, int max_seq, int pdl,
                        void* stream);

/* Workspace bytes w4_lm_head_argmax needs (zeroed once by the caller). */
size_t w4_lm_head_workspace_bytes(void);

/* w4_lm_head_argmax: x = rmsnorm(h) * norm_weight, logits[v] = embed[v, :]
 * . x (bf16, the tied embedding as lm_head), token <- argmax (first index
 * among equal bf16 logits, like torch.argmax), pos <- pos + 1. logits may be
 * NULL. hidden is one of 256, 512, 1024, 1536, 2048. The workspace (w4_lm_head_workspace_bytes, zeroed before the first
 * call) carries the cross-CTA argmax and is left zeroed again. */
int w4_lm_head_argmax(const void* h, const void* norm_weight, float eps,
                      const void* embed, int vocab, int hidden, void* logits,
                      int64_t* token, int64_t* pos, void* workspace,
                      size_t workspace_bytes, int pdl, void* stream);

/* w4_lm_head_argmax for hosts that cannot allocate device memory. There is
 * no counterpart of this entry point in the reference.
 *
 * Some callers of this library may not allocate: a C or C++ decode loop in
 * a process whose device memory belongs to another runtime's pool, or a
 * plugin that must not call an allocator once it is serving. This variant
 * needs no workspace: the argmax state lives in a 256-byte array inside the
 * library's module, present on every GPU that loads the library until the
 * process exits. It allocates and frees nothing. Its first call on a device
 * looks up that array's address and clears it on the given stream, so make
 * that first call before any stream capture. The address is kept per device
 * for the life of the process; it does not survive cudaDeviceReset, after
 * which this entry point must not be called again in the same process. All
 * calls on a device share the one array: calls that overlap on the GPU race.
 * The array (W4B200_STATIC_SCRATCH_BYTES) holds the same few words of argmax
 * state whatever the vocab, so there is no vocab limit beyond a positive int
 * (W4B200_STATIC_SCRATCH_MAX_VOCAB is that bound, given for information);
 * hidden is checked against the built sizes before the array is touched.
 * Other arguments as w4_lm_head_argmax. */
#define W4B200_STATIC_SCRATCH_BYTES 256
#define W4B200_STATIC_SCRATCH_MAX_VOCAB 0x7fffffff
int w4_lm_head_argmax_static(const void* h, const void* norm_weight, float eps,
                             const void* embed, int vocab, int hidden,
                             void* logits, int64_t* token, int64_t* pos,
                             int pdl, void* stream);

/* ---------------------------------------------------------------------
 * The whole decode step as one persistent kernel.
 *
 * Replaces the per-token model forward of scripts/decode_loop.py:106-124
 * (HF forward + argmax + .item()) with one cooperative launch per token:
 * embedding, every layer (RMSNorm, q|k|v, RoPE, KV write, attention, o,
 * RMSNorm, gate|up, SwiGLU, down, residuals), final RMSNorm, tied lm_head
 * and argmax. The int4 weights use the reference packing
 * (src/roofline/kernels.py:24-47) stacked over layers: packed
 * [layers * K/8, N], scales [layers * K/128, N]. All other tensors are bf16.
 * Needs head_dim 128, heads / kv_heads <= 8 and hidden in {256, 512, 1024,
 * 1536, 2048}. */
typedef struct w4_decode_model {
  int layers, hidden, intermediate, heads, kv_heads, head_dim, vocab, max_seq;
  float eps;                       /* RMSNorm epsilon */
  const int32_t* qkv_packed;       /* [layers*hidden/8, hidden + 2*kv_heads*128] */
  const void* qkv_scales;
  const int32_t* o_packed;         /* [layers*hidden/8, hidden] */
  const void* o_scales;
  const int32_t* gu_packed;        /* [layers*hidden/8, 2*intermediate] (gate | up) */
  const void* gu_scales;
  const int32_t* down_packed;      /* [layers*intermediate/8, hidden] */
  const void* down_scales;
  const void* qkv_bias;            /* [layers, hidden + 2*kv_heads*128] */
  const void* in_norm;             /* [layers, hidden] */
  const void* post_norm;           /* [layers, hidden] */
  const void* final_norm;          /* [hidden] */
  const void* embed;               /* [vocab, hidden], also the lm_head */
  const void* cos_table;           /* [max_seq, 128] */
  const void* sin_table;           /* [max_seq, 128] */
  void* k_cache;                   /* [layers, kv_heads, max_seq, 128] */
  void* v_cache;
  const int64_t* prompt;           /* prompt ids; position p < *prompt_len reads prompt[p] */
  const int64_t* prompt_len;
  int64_t* token;                  /* in: previous argmax; out: this step's argmax */
  int64_t* pos;                    /* in: position of this step; out: pos + 1 */
  void* logits;                    /* [vocab] bf16, may be NULL */
} w4_decode_model;

/* Bytes of device scratch w4_decode_step needs for this model on the
 * current device (zeroed once by the caller, 256-byte aligned). */
int w4_decode_step_scratch_bytes(const w4_decode_model* model, size_t* bytes);

/* One greedy decode step. The step's grid barriers are bounded waits: if one
 * gives up, w4_device_error reports it and the scratch must be zeroed again
 * before the next step. */
int w4_decode_step(const w4_decode_model* model, void* scratch, size_t scratch_bytes,
                   void* stream);

/* Reads and clears the device-side error word that kernels set when a
 * bounded wait gives up (0 = no error). Synchronises the device. */
int w4_device_error(int device, int* code);

#ifdef __cplusplus
}
#endif

#endif /* W4B200_H_ */
