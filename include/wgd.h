/*
 * wgd — B200-native decoder loop for GGUF models: C ABI.
 *
 * This library is the device half of the reference runtime's PagedEngine
 * (ahpah-dev/WebGPU 0.9.0): it replaces the WebGPU `Compute` wrapper
 * (src/core/gpu.ts:2-67), the page uploads of `WeightPager`
 * (src/core/pager.ts:7-47) and the per-layer dispatch sequence of
 * `PagedEngine.forward/denseLayer/linear` (src/core/engine.ts:117-256).
 * GGUF parsing, tokenizers and the SDK/worker protocol stay in the host
 * language and call these entry points.
 *
 * Conventions
 *   - Every call returns WGD_OK (0) or a WGD_E* status; the message of the last
 *     failure on the calling thread is wgd_last_error().
 *   - Host buffers are borrowed for the duration of a call. Device memory is
 *     owned by the context and counted against its byte budget, with the same
 *     meaning as the reference's GPU budget (gpu.ts:10,23-30).
 *   - One calling thread per context; wgd_cancel() is the only call that is safe
 *     from another thread.
 *   - The wgd_op_* entry points run one kernel on caller-owned DEVICE pointers
 *     (the reference's per-kernel checks in src/verify.ts and
 *     src/verify-context.ts exercise the same kernels one at a time).
 */
#ifndef WGD_H
#define WGD_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WGD_ABI_VERSION 1

#if defined(__GNUC__)
#define WGD_API __attribute__((visibility("default")))
#else
#define WGD_API
#endif

enum wgd_status {
  WGD_OK = 0,
  WGD_EINVAL = 1,       /* bad argument or unsupported shape */
  WGD_EBUDGET = 2,      /* device budget exceeded (gpu.ts:25) */
  WGD_ECUDA = 3,        /* CUDA runtime or kernel error */
  WGD_ECANCELLED = 4,   /* wgd_cancel() observed (engine.ts:128,147 AbortSignal checks) */
  WGD_ETIMEOUT = 5,     /* a bounded wait on a tensor-parallel peer gave up */
  WGD_ESTATE = 6,       /* call out of order (e.g. forward before all weights are uploaded) */
  WGD_ENONFINITE = 7,   /* every logit was non-finite (engine.ts:308) */
  WGD_EIO = 8           /* the page reader callback failed */
};

/* GGML tensor types the reference decodes (QUANTS, gguf.ts:6-11; decodeWeight, quant.ts:6-29). */
enum wgd_ggml_type { WGD_F32 = 0, WGD_F16 = 1, WGD_Q4_0 = 2, WGD_Q8_0 = 8, WGD_Q4_K = 12, WGD_Q5_K = 13, WGD_Q6_K = 14 };

/* Decoder configuration; mirrors ModelConfig (src/core/gguf.ts:87-107) as
 * produced by modelConfig (gguf.ts:108-213). */
typedef struct wgd_model_config {
  int32_t family;          /* 0: dense llama/qwen2/qwen3/mistral block, 1: gemma3 block */
  int32_t hidden, intermediate, layers, heads, kv_heads, head_dim, vocab;
  float epsilon, theta, local_theta;
  int32_t window, period;  /* gemma3 local window and layer period (gguf.ts:131,133) */
  float attention_scale, rope_scale;
  int32_t rotary_dim;
  int32_t rope_mode;       /* 0: half-split (neox), 1: adjacent pairs (norm) (gguf.ts:139) */
  int32_t sliding_window;  /* dense families: 0 = full context (gguf.ts:140) */
  int32_t qk_norm, ffn_gate, activation; /* activation 0: silu, 1: gelu */
  int32_t bias_q, bias_k, bias_v, bias_output;
} wgd_model_config;

/* PagingStats (src/core/pager.ts:5) plus device timings. */
typedef struct wgd_stats {
  uint64_t read_bytes, uploads, cache_hits, cache_bytes, gpu_bytes, peak_gpu_bytes, page_bytes;
  double read_ms;
  uint64_t forwards, tokens;
  double last_forward_ms;   /* device time of the last forward (CUDA events) */
  uint64_t streamed_bytes;  /* weight bytes streamed through page slots by the last forward */
  uint64_t kernel_launches; /* kernels this library launched for forwards and decodes, cumulative */
} wgd_stats;

typedef struct wgd_ctx wgd_ctx;

/* Reads `length` bytes at `offset` of the model file into `dst` (a pinned
 * staging buffer owned by the library). Returns 0 on success. Mirrors
 * ByteSource.read (src/core/source.ts:2-6). */
typedef int (*wgd_read_fn)(void *user, uint64_t offset, uint64_t length, void *dst);

WGD_API int wgd_abi_version(void);
WGD_API const char *wgd_last_error(void);
WGD_API int wgd_device_count(int *count);

/* Context on one GPU; replaces Compute.init (gpu.ts:11-21) and the budget
 * (gpu.ts:10). tp_rank/tp_size place this process in a tensor-parallel group
 * (one process per GPU); page_bytes is the pager's page size (pager.ts:15-19). */
WGD_API wgd_ctx *wgd_create(int device, int tp_rank, int tp_size, uint64_t budget_bytes, uint32_t page_bytes, int *status);
WGD_API void wgd_destroy(wgd_ctx *ctx);

/* Tensor-parallel wiring (no counterpart in the reference, which runs on one
 * device). Each rank exports a handle to its exchange buffer; the host
 * exchanges the handles (e.g. through torch.distributed) and opens the peers'. */
WGD_API int wgd_tp_handle_size(void);
WGD_API int wgd_tp_export(wgd_ctx *ctx, void *handle_out);
WGD_API int wgd_tp_open_peers(wgd_ctx *ctx, const void *handles /* tp_size * handle_size bytes, rank order */);
/* Bounded wait (iterations) for peers in the exchange kernel; 0 = default. */
WGD_API int wgd_tp_set_timeout(wgd_ctx *ctx, uint64_t spin_limit);

/* Model setup; replaces PagedEngine.load's allocation half (engine.ts:70-110).
 * Order: model_begin, tensor_register for each directory entry, model_end,
 * tensor_upload (or tensor_host / page reader for streamed weights). */
WGD_API int wgd_model_begin(wgd_ctx *ctx, const wgd_model_config *cfg, int context_len, int max_batch);
/* One entry of the GGUF tensor directory (Tensor, gguf.ts:4; dims in GGUF order). */
WGD_API int wgd_tensor_register(wgd_ctx *ctx, const char *name, int ggml_type, const uint64_t *dims, int nd,
                        uint64_t file_offset, uint64_t bytes, uint64_t row_bytes);
WGD_API int wgd_model_end(wgd_ctx *ctx);
/* Uploads bytes [byte_off, byte_off+n) of a tensor's GGUF data (whole rows); replaces
 * WeightPager.page + Compute.write (pager.ts:25-44). model_end decides where each matrix lives:
 * on the device while the budget allows (less a 16 MiB margin), otherwise in pinned host memory
 * owned by the library, from which every forward streams it page by page (page_bytes, two device
 * slots, a copy stream); the data is repacked into the device layout either way. */
WGD_API int wgd_tensor_upload(wgd_ctx *ctx, const char *name, uint64_t byte_off, const void *host, uint64_t n);
/* Uploads a whole tensor from `host` (all of its GGUF bytes; the memory is read during the call
 * only). `pinned` is a hint that the memory is page-locked. */
WGD_API int wgd_tensor_host(wgd_ctx *ctx, const char *name, const void *host, int pinned);
/* Sets the byte-range reader wgd_load_weights pulls the model through (ByteSource.read,
 * source.ts:2-6): reads of at most page_bytes (whole rows) into a library-owned buffer. */
WGD_API int wgd_set_page_reader(wgd_ctx *ctx, wgd_read_fn fn, void *user);
/* Uploads every tensor this rank needs through the page reader (after model_end). */
WGD_API int wgd_load_weights(wgd_ctx *ctx);
/* 1 if every weight needed by forward is resident or has a stream source. */
WGD_API int wgd_model_ready(wgd_ctx *ctx, int *ready);
/* Resident weight bytes and streamed weight bytes of the placement plan. */
WGD_API int wgd_model_placement(wgd_ctx *ctx, uint64_t *resident_bytes, uint64_t *streamed_bytes);
/* The residency rule wgd_model_end applies, as a pure host function (no device
 * calls): for n matrices of sizes[i] device bytes (whole 256-byte units, in
 * execution order) placed after `allocated` bytes under `budget`, resident[i]
 * is 1 for the matrices kept on the device and 0 for those streamed through
 * the two page slots, whose size goes to *slot_bytes (0 when nothing streams).
 * Replaces the cache/stream decision of the WeightPager class (src/core/pager.ts:22,37-41:
 * a resident prefix while cacheBudget = limit - allocated - 16 MiB allows,
 * then one streaming slot). */
WGD_API int wgd_plan_residency(const uint64_t *sizes, int n, uint64_t allocated, uint64_t budget, uint64_t page_bytes,
                               uint64_t unit_max, int32_t *resident, uint64_t *slot_bytes);

/* One forward over n token ids at positions [start, start+n); replaces
 * PagedEngine.forward (engine.ts:138-180). want: 0 no output, 1 greedy token
 * of the last row (engine.ts:305-309), 2 greedy token and full logits of the
 * last row (vocab floats, rank 0 of a TP group). */
WGD_API int wgd_forward(wgd_ctx *ctx, const int32_t *ids, int n, int start, int want, int32_t *argmax_out, float *logits_out);
/* Greedy decode of `steps` tokens entirely on the device: `first` is the token
 * at position `start`; each step's argmax becomes the next step's input
 * without a host round trip (the reference's greedy generate loop,
 * engine.ts:290-297, with sample() on the device). tokens_out receives the
 * `steps` generated ids (stopping early is the caller's business). */
WGD_API int wgd_decode(wgd_ctx *ctx, int32_t first, int start, int steps, int32_t *tokens_out);
/* One forward (as wgd_forward) and a draw from the last row's logits on the device, replacing the
 * logits readback and sample() of PagedEngine.generate (engine.ts:291,305-324): top_k candidates by
 * value (lower index first among equal values), p = exp((v - best) / temperature), the nucleus cut
 * at top_p, draw = uniform * retained mass. `uniform` in [0, 1) takes the place of Math.random().
 * Settings follow GenerationOptions (engine.ts:21,264): temperature in [0, 2] (0 = greedy), top_k
 * 1..200, top_p in (0, 1]; otherwise WGD_EINVAL "Invalid sampling settings.". No finite logit:
 * WGD_ENONFINITE. Under tensor parallelism every rank draws the same token (the logits are gathered). */
WGD_API int wgd_forward_sample(wgd_ctx *ctx, const int32_t *ids, int n, int start, double temperature, int top_k, double top_p,
                               double uniform, int32_t *token_out);
/* wgd_decode with the same draw in place of the argmax: step i uses uniforms[i]; each drawn token
 * is the next step's input without a host round trip. */
WGD_API int wgd_decode_sample(wgd_ctx *ctx, int32_t first, int start, int steps, double temperature, int top_k, double top_p,
                              const double *uniforms, int32_t *tokens_out);
/* Kernels launched by the last forward (per token) or persistent call (1), for launch accounting. */
WGD_API int wgd_kernels_per_token(wgd_ctx *ctx, int *count);
/* KV cache bookkeeping for prefix reuse and reset (engine.ts:269-283,302). */
WGD_API int wgd_truncate_kv(wgd_ctx *ctx, int n_tokens);
WGD_API void wgd_cancel(wgd_ctx *ctx);
WGD_API int wgd_stats_get(wgd_ctx *ctx, wgd_stats *out);
/* Enables/disables CUDA-graph replay of single-token forwards (default on). */
WGD_API int wgd_set_graphs(wgd_ctx *ctx, int enabled);
/* Enables/disables the persistent decode kernel (default on): single-row forwards and wgd_decode
 * then run as one cooperative launch per call (all layers, LM head, argmax, token feedback) when the
 * model's shapes allow it; otherwise, or when disabled, they use the per-kernel path. */
WGD_API int wgd_set_persistent(wgd_ctx *ctx, int enabled);
/* Projections of Q4_K/Q6_K matrices for forward batches of at least min_batch rows run on the tcgen05
 * tensor-core GEMM (wgd_op_gemm_tiled) instead of the GEMV; 0 turns it off. Default 16; takes
 * effect only if the model was loaded with a batch size of 8 or more. */
WGD_API int wgd_set_prefill_gemm(wgd_ctx *ctx, int min_batch);
/* 1 when the persistent decode kernel is available for this model, 0 when not (the reason is
 * written to why[0..why_len)). */
WGD_API int wgd_persistent_status(wgd_ctx *ctx, char *why, int why_len);

/* ---------------------------------------------------------------- kernels
 * Single-kernel entry points on caller-owned device memory, on `stream`
 * (a cudaStream_t, or NULL for the legacy default stream). They allocate
 * small per-device scratch (work counters) on first use. */

/* The draw of wgd_forward_sample over n fp32 logits in device memory; the token is written to host
 * memory (the call waits for it). */
WGD_API int wgd_op_sample(const float *logits, int n, double temperature, int top_k, double top_p, double uniform,
                          int32_t *token_out, void *stream);
/* Bytes of one row in the device layout used by every weight kernel. */
WGD_API int64_t wgd_dev_row_bytes(int ggml_type, int64_t cols);
/* GGUF rows (raw bytes, row stride gguf row bytes) -> device layout rows. */
WGD_API int wgd_op_repack(int ggml_type, int64_t rows, int64_t cols, const void *raw_dev, void *packed_dev, void *stream);
/* Bit-exact dequant (WGSL f32 expression order, weightFunction, shaders.ts:13-38) of packed rows. */
WGD_API int wgd_op_dequant(int ggml_type, int64_t rows, int64_t cols, const void *packed_dev, float *out_dev, void *stream);
/* y[b*rows + r] = sum_c W[r][c] * x[b*cols + c] for b < batch (matmulShader,
 * shaders.ts:39-54; expectation verify.ts:32-35). */
WGD_API int wgd_op_gemv(int ggml_type, int64_t rows, int64_t cols, const void *packed_dev, const float *x_dev, int batch,
                float *y_dev, void *stream);
/* Tile-16 layout used by the tensor-core GEMV for Q4_K / Q6_K matrices (rows
 * in groups of 16, each GGUF block column of a group stored together so that
 * mma.sync fragments load with coalesced 16-byte reads). Bytes of a rows x
 * cols matrix, or -1 if the type/shape has no tiled form. */
WGD_API int64_t wgd_tiled_bytes(int ggml_type, int64_t rows, int64_t cols);
WGD_API int wgd_op_repack_tiled(int ggml_type, int64_t rows, int64_t cols, const void *raw_dev, void *tiled_dev, void *stream);
WGD_API int wgd_op_dequant_tiled(int ggml_type, int64_t rows, int64_t cols, const void *tiled_dev, float *out_dev, void *stream);
/* The same product as wgd_op_gemv over tiled weights (integer tensor-core path). */
WGD_API int wgd_op_gemv_tiled(int ggml_type, int64_t rows, int64_t cols, const void *tiled_dev, const float *x_dev, int batch,
                              float *y_dev, void *stream);
/* wgd_op_gemv_tiled for callers that may not allocate device memory while running (no counterpart in
 * the reference, whose WebGPU path has no such constraint): the scratch is a fixed per-device array of
 * 4 MiB of partial sums and 8192 tile counters, and shapes needing more fail with WGD_EINVAL. The first
 * call on a device (that device current) looks the scratch up and should come before any stream capture;
 * no call allocates. The looked-up address is kept for the life of the process, so the device's CUDA
 * context must not be reset in between. Calls on one device must not overlap in time: they share the
 * scratch. */
WGD_API int wgd_op_gemv_tiled_noalloc(int ggml_type, int64_t rows, int64_t cols, const void *tiled_dev, const float *x_dev,
                                      int batch, float *y_dev, void *stream);
/* Prompt-batch product over tiled Q4_K / Q6_K weights on the tcgen05 tensor cores (the matmul shader,
 * shaders.ts, for a batch of rows; engine.ts:217-251 runs it for every projection of a prefill
 * batch): y[b * rows + r] = sum_c W[r][c] * x[b * cols + c] for b < batch, 1 <= batch <= 128.
 * Weights exact in f16, activations split into two f16 terms, f32 accumulation: the result
 * agrees with wgd_op_gemv_tiled to fp32 rounding. Asynchronous on `stream`;
 * wgd_op_gemm_tiled_status reports (and clears) a pipeline wait that ran out on this device. */
WGD_API int wgd_op_gemm_tiled(int ggml_type, int64_t rows, int64_t cols, const void *tiled_dev, const float *x_dev, int batch,
                              float *y_dev, void *stream);
WGD_API int wgd_op_gemm_tiled_status(int *status);
/* RMSNorm of n rows (normShader, shaders.ts:55-68). */
WGD_API int wgd_op_rmsnorm(const float *x_dev, const float *w_dev, int cols, int n, float eps, float *y_dev, void *stream);
/* Q/K rotation (+ optional per-head RMS norm) of x[n][heads][hd] in place:
 * ropeShader / ropeNeoxShader / ropeClassicShader (shaders.ts:69-87,139-154,155-169).
 * mode 0 half-split, 1 adjacent; norm_w non-null selects the Q/K-norm form. */
WGD_API int wgd_op_rope(float *x_dev, const float *norm_w_dev, int n, int heads, int hd, int start, float theta, float scale,
                float eps, int rotary_dim, int mode, void *stream);
/* Causal GQA attention over a ring cache laid out [kv_heads][capacity][hd]
 * (attentionShader, shaders.ts:88-122). q/out are [n][heads][hd]. */
WGD_API int wgd_op_attention(const float *q_dev, const float *k_dev, const float *v_dev, float *out_dev, int n, int heads,
                     int kv_heads, int hd, int start, float scale, int window, int capacity, void *stream);
/* First finite maximum of x[0..n) (engine.ts:305-309); *idx_dev = -1 when none. */
WGD_API int wgd_op_argmax(const float *x_dev, int n, int32_t *idx_dev, void *stream);

#ifdef __cplusplus
}
#endif
#endif
