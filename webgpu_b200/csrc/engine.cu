// The decoder engine behind include/wgd.h.
//
// One wgd_ctx owns one GPU (one process per GPU for tensor parallelism). The
// per-token sequence follows PagedEngine.forward / denseLayer and the Gemma
// block of the reference (src/core/engine.ts:138-180, 158-174, 217-251), with
// its dispatches fused:
//   embed -> per layer [ QKV GEMV (+attn RMSNorm prologue, +bias)
//                        -> Q/K-norm + RoPE + KV ring write
//                        -> split-K attention
//                        -> O GEMV (+residual, or post-norm for Gemma)
//                        -> gate|up GEMV (+ffn RMSNorm prologue, +SwiGLU/GeGLU)
//                        -> down GEMV (+residual, or post-norm) ]
//          -> LM head GEMV (+output RMSNorm prologue) on the last row -> argmax.
// Single-token forwards are captured once into a CUDA graph (positions live in
// device memory, so one graph serves every step) and replayed.
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/wgd.h"
#include "common.cuh"
#include "kernels.h"
#include "persist.h"
#include "tile.cuh"
#include "tp.h"

using namespace wgd;

static thread_local std::string g_err;
static int fail(int code, const std::string &msg) {
  g_err = msg;
  return code;
}
namespace wgd {
// Sets the thread's wgd_last_error() text for entry points defined in other files.
int api_fail(int code, const std::string &msg) { return fail(code, msg); }
}  // namespace wgd
#define CK(call)                                                                                  \
  do {                                                                                            \
    cudaError_t e_ = (call);                                                                      \
    if (e_ != cudaSuccess) return fail(WGD_ECUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)

namespace {

struct DevLinear {
  int type = -1, rows = 0, cols = 0, nb = 0;
  int64_t drow = 0;       // row layout: bytes per row
  bool tiled = false;     // tile-16 layout (tensor-core GEMV)
  bool streamed = false;  // kept in pinned host memory and paged through device slots per forward
  int unit_rows = 1;      // page granularity in rows (a tile, or a gate|up interleave block)
  uint8_t *w = nullptr;   // device pointer (a mapped host pointer when streamed)
  const char *label = "";
  int64_t bytes() const { return tiled ? tiled_bytes(type, rows, cols) : drow * rows; }
  int64_t unit_bytes() const { return tiled ? (int64_t)(cols / 256) * tile_chunk_bytes(type) : drow * unit_rows; }
};

enum Role {
  R_NONE, R_EMBD, R_OUT_NORM, R_OUTPUT, R_ATTN_NORM, R_Q, R_K, R_V, R_O, R_QB, R_KB, R_VB, R_OB, R_QN, R_KN,
  R_POST_ATTN, R_FFN_NORM, R_GATE, R_UP, R_DOWN, R_POST_FFW
};
struct RoleName { const char *name; Role role; };
const RoleName LAYER_ROLES[] = {
  {"attn_norm.weight", R_ATTN_NORM}, {"attn_q.weight", R_Q}, {"attn_k.weight", R_K}, {"attn_v.weight", R_V},
  {"attn_output.weight", R_O}, {"attn_q.bias", R_QB}, {"attn_k.bias", R_KB}, {"attn_v.bias", R_VB},
  {"attn_output.bias", R_OB}, {"attn_q_norm.weight", R_QN}, {"attn_k_norm.weight", R_KN},
  {"post_attention_norm.weight", R_POST_ATTN}, {"ffn_norm.weight", R_FFN_NORM}, {"ffn_gate.weight", R_GATE},
  {"ffn_up.weight", R_UP}, {"ffn_down.weight", R_DOWN}, {"post_ffw_norm.weight", R_POST_FFW}};

struct TensorRec {
  std::string name;
  int type = 0, nd = 0;
  uint64_t dims[4] = {0, 0, 0, 0};
  uint64_t offset = 0, bytes = 0, row_bytes = 0;
  int64_t cols = 0, rows = 0;
  int layer = -1;
  Role role = R_NONE;
  // destination of a matrix
  DevLinear *lin = nullptr;
  RowMap map{};
  int blk0 = 0, nbl = 0;
  // destination of a vector: elements [vec_src0, vec_src0 + vec_len) -> vec
  float *vec = nullptr;
  int vec_src0 = 0, vec_len = 0;
  int64_t uploaded_rows = 0;
  bool needed = false;
  const void *host = nullptr;
};

struct Layer {
  float *attn_norm = nullptr, *qkv_bias = nullptr, *q_norm = nullptr, *k_norm = nullptr, *o_bias = nullptr;
  float *post_attn = nullptr, *ffn_norm = nullptr, *post_ffw = nullptr;
  DevLinear qkv, o, gate_up, down;
  float *k_cache = nullptr, *v_cache = nullptr;
  int capacity = 0, window = 0;
  bool local = false;
  double theta = 0, rope_scale = 1;
  const float2 *rope_table = nullptr;  // (cos, sin)[context][rot/2] for this layer's theta/scale
};

struct Alloc { void *p; size_t n; };

}  // namespace

struct wgd_ctx {
  int device = 0, tp_rank = 0, tp_size = 1, sm_count = 148;
  uint64_t budget = 0, allocated = 0, peak = 0;
  uint32_t page_bytes = 16u << 20;
  cudaStream_t stream = nullptr;
  std::vector<Alloc> allocs;
  // model
  bool begun = false, ended = false;
  wgd_model_config c{};
  int context = 0, max_batch = 0;
  std::vector<TensorRec> tensors;
  std::unordered_map<std::string, int> by_name;
  int heads_l = 0, kv_l = 0, q_l = 0, kvd_l = 0, qkv_rows = 0, ffn0 = 0, ffn_l = 0, vocab0 = 0, vocab_l = 0;
  std::vector<Layer> layers;
  DevLinear embd, lm;
  float *out_norm = nullptr;
  bool tied = false;
  // work buffers
  float *hidden = nullptr, *qkv = nullptr, *qrot = nullptr, *att = nullptr, *proj = nullptr, *act = nullptr, *logits = nullptr;
  int *d_ids = nullptr, *d_start = nullptr, *d_argmax = nullptr, *d_err = nullptr;
  float *d_maxval = nullptr, *att_part = nullptr, *am_part = nullptr;
  unsigned *att_ctr = nullptr, *am_ctr = nullptr;
  int att_splits = 1;
  uint8_t *staging = nullptr;
  size_t staging_bytes = 0;
  std::vector<std::pair<std::pair<double, double>, float2 *>> rope_tables;  // (theta, scale) -> table
  float *g2_part = nullptr;  // stream-K partials of the tensor-core GEMV
  size_t g2_part_floats = 0;
  unsigned *g2_ctr = nullptr;
  int g2_ctr_count = 0;
  // prompt-batch tcgen05 GEMM (gemm_tc.cu): Q4_K/Q6_K projections of batches >= tc_min_batch
  int tc_min_batch = 16;
  int tc_cols_max = 0, tc_rows_max = 0;
  uint8_t *tc_panel = nullptr;
  float *tc_part = nullptr;
  unsigned *tc_ctr = nullptr;
  int *tc_status = nullptr;  // device address of h_io[IO_TC]
  // device sampling (sample.cu): settings, per-step uniforms [context], CTA keys, counter
  SampleParams *d_sparams = nullptr;
  double *d_uniform = nullptr;
  uint64_t *smp_part = nullptr;
  unsigned *smp_ctr = nullptr;
  int *d_ptok = nullptr;  // token slot of the persistent kernel when the draw replaces its argmax
  int32_t *h_io = nullptr;  // pinned: [0] start, [1] argmax, [2..] ids
  // graph
  bool graphs = true;
  cudaGraphExec_t decode_exec = nullptr, chain_exec = nullptr, chain_smp_exec = nullptr;
  cudaGraph_t decode_graph = nullptr, chain_graph = nullptr, chain_smp_graph = nullptr;
  int *d_tokens = nullptr, *d_step = nullptr;
  int kernels = 0;  // kernels launched by the last enqueued forward
  int decode_kernels = 0, chain_kernels = 0, chain_smp_kernels = 0;  // kernels in the captured graphs
  std::atomic<int> cancel{0};
  wgd_stats st{};
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  TpComm *tp = nullptr;
  uint64_t tp_spin_limit = 0;
  // persistent decode kernel (one launch per wgd_forward of one row / per wgd_decode)
  bool persist_ok = false, persist_on = true;
  std::string persist_why = "not built";
  PersistArgs pargs{};
  int *h_status = nullptr;  // pinned mirror of pargs.status
  // tensor-parallel persistent launches: arrivals on this rank's cross-rank counter and tokens
  // decoded so far (identical on every rank of the group); a wait that ran out breaks the group
  unsigned x_arrivals = 0, x_tokens = 0;
  bool tp_broken = false;
  // weight pager (WeightPager, pager.ts): matrices that do not fit the budget live in pinned host
  // memory and stream through two device page slots on a copy stream
  std::vector<DevLinear *> pending;  // matrices placed by model_end, in execution order
  std::vector<void *> host_allocs;
  bool paging = false;
  uint8_t *slot[2] = {nullptr, nullptr};
  size_t slot_bytes = 0;
  cudaStream_t copy_stream = nullptr;
  cudaEvent_t copied[2] = {nullptr, nullptr}, freed[2] = {nullptr, nullptr};
  unsigned page_seq = 0;
  wgd_read_fn reader = nullptr;  // ByteSource.read for wgd_load_weights
  void *reader_user = nullptr;
  uint8_t *reader_buf = nullptr;
  uint64_t reader_buf_bytes = 0;
};
// h_io slots: [0] start, [1] argmax, [2..1015] ids, [1016..1019] persistent status, [1020] cancel word,
// [1021] tensor-core GEMM status
constexpr int IO_STATUS = 1016, IO_CANCEL = 1020, IO_TC = 1021;

// ------------------------------------------------------------------ helpers

static int ctx_alloc(wgd_ctx *ctx, void **p, size_t n, const char *label) {
  n = (size_t)align_up((int64_t)(n ? n : 4), 256);
  if (ctx->allocated + n > ctx->budget)
    return fail(WGD_EBUDGET, std::string("GPU budget exceeded. Reduce context length or increase the memory budget. (") +
                                 label + ")");
  cudaError_t e = cudaMalloc(p, n);
  if (e != cudaSuccess) return fail(WGD_ECUDA, std::string("cudaMalloc(") + label + "): " + cudaGetErrorString(e));
  e = cudaMemset(*p, 0, n);
  if (e != cudaSuccess) return fail(WGD_ECUDA, std::string("cudaMemset: ") + cudaGetErrorString(e));
  ctx->allocs.push_back({*p, n});
  ctx->allocated += n;
  if (ctx->allocated > ctx->peak) ctx->peak = ctx->allocated;
  return WGD_OK;
}
template <typename T>
static int ctx_alloc_t(wgd_ctx *ctx, T **p, size_t count, const char *label) {
  void *v = nullptr;
  int rc = ctx_alloc(ctx, &v, count * sizeof(T), label);
  *p = (T *)v;
  return rc;
}

static void free_all(wgd_ctx *ctx) {
  if (ctx->decode_exec) cudaGraphExecDestroy(ctx->decode_exec);
  if (ctx->decode_graph) cudaGraphDestroy(ctx->decode_graph);
  if (ctx->chain_exec) cudaGraphExecDestroy(ctx->chain_exec);
  if (ctx->chain_graph) cudaGraphDestroy(ctx->chain_graph);
  if (ctx->chain_smp_exec) cudaGraphExecDestroy(ctx->chain_smp_exec);
  if (ctx->chain_smp_graph) cudaGraphDestroy(ctx->chain_smp_graph);
  ctx->decode_exec = ctx->chain_exec = ctx->chain_smp_exec = nullptr;
  ctx->decode_graph = ctx->chain_graph = ctx->chain_smp_graph = nullptr;
  for (auto &a : ctx->allocs) cudaFree(a.p);
  ctx->allocs.clear();
  ctx->allocated = 0;
  for (void *h : ctx->host_allocs) cudaFreeHost(h);
  ctx->host_allocs.clear();
  ctx->pending.clear();
}

static bool parse_layer_name(const std::string &name, int &layer, Role &role) {
  if (name.compare(0, 4, "blk.") != 0) return false;
  size_t dot = name.find('.', 4);
  if (dot == std::string::npos) return false;
  layer = atoi(name.substr(4, dot - 4).c_str());
  std::string rest = name.substr(dot + 1);
  for (const auto &r : LAYER_ROLES)
    if (rest == r.name) { role = r.role; return true; }
  role = R_NONE;
  return true;
}

// Balanced split of `units` into tp parts: part r = [r*units/tp, (r+1)*units/tp).
static int part_begin(int units, int r, int tp) { return (int)((int64_t)units * r / tp); }

// ------------------------------------------------------------------ C ABI

extern "C" {

int wgd_abi_version(void) { return WGD_ABI_VERSION; }
const char *wgd_last_error(void) { return g_err.c_str(); }

int wgd_device_count(int *count) {
  if (!count) return fail(WGD_EINVAL, "count is null");
  CK(cudaGetDeviceCount(count));
  return WGD_OK;
}

wgd_ctx *wgd_create(int device, int tp_rank, int tp_size, uint64_t budget_bytes, uint32_t page_bytes, int *status) {
  auto set = [&](int s) { if (status) *status = s; };
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
    set(fail(WGD_EINVAL, "invalid CUDA device"));
    return nullptr;
  }
  if (tp_size < 1 || tp_size > 8 || tp_rank < 0 || tp_rank >= tp_size) {
    set(fail(WGD_EINVAL, "tensor-parallel size must be 1-8 and rank within it"));
    return nullptr;
  }
  if (page_bytes != (16u << 20) && page_bytes != (64u << 20)) {
    set(fail(WGD_EINVAL, "Weight pages must be 16 or 64 MiB."));
    return nullptr;
  }
  if (cudaSetDevice(device) != cudaSuccess) { set(fail(WGD_ECUDA, "cudaSetDevice failed")); return nullptr; }
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major < 10) {
    set(fail(WGD_EINVAL, "wgd requires a Blackwell (sm_100) GPU"));
    return nullptr;
  }
  auto *ctx = new wgd_ctx();
  ctx->device = device;
  ctx->tp_rank = tp_rank;
  ctx->tp_size = tp_size;
  ctx->budget = budget_bytes;
  ctx->page_bytes = page_bytes;
  ctx->sm_count = prop.multiProcessorCount;
  if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreate(&ctx->ev0) != cudaSuccess || cudaEventCreate(&ctx->ev1) != cudaSuccess ||
      cudaMallocHost((void **)&ctx->h_io, sizeof(int32_t) * 1024) != cudaSuccess) {
    set(fail(WGD_ECUDA, "stream/event/pinned allocation failed"));
    delete ctx;
    return nullptr;
  }
  memset(ctx->h_io, 0, sizeof(int32_t) * 1024);
  ctx->st.page_bytes = page_bytes;
  set(WGD_OK);
  return ctx;
}

void wgd_destroy(wgd_ctx *ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  if (ctx->copy_stream) cudaStreamSynchronize(ctx->copy_stream);
  if (ctx->tp) tp_destroy(ctx->tp);
  free_all(ctx);
  if (ctx->h_io) cudaFreeHost(ctx->h_io);
  if (ctx->reader_buf) cudaFreeHost(ctx->reader_buf);
  if (ctx->ev0) cudaEventDestroy(ctx->ev0);
  if (ctx->ev1) cudaEventDestroy(ctx->ev1);
  for (int i = 0; i < 2; i++) {
    if (ctx->copied[i]) cudaEventDestroy(ctx->copied[i]);
    if (ctx->freed[i]) cudaEventDestroy(ctx->freed[i]);
  }
  if (ctx->copy_stream) {
    cudaStreamSynchronize(ctx->copy_stream);
    cudaStreamDestroy(ctx->copy_stream);
  }
  if (ctx->stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
}

int wgd_model_begin(wgd_ctx *ctx, const wgd_model_config *cfg, int context_len, int max_batch) {
  if (!ctx || !cfg) return fail(WGD_EINVAL, "null argument");
  if (ctx->begun) return fail(WGD_ESTATE, "model already configured");
  const wgd_model_config &c = *cfg;
  // ModelConfig validation (gguf.ts:149) plus what the kernels need.
  if (c.layers < 1 || c.hidden < 1 || c.heads < 1 || c.head_dim < 1 || c.kv_heads < 1 || c.intermediate < 1 ||
      c.vocab < 1 || c.heads % c.kv_heads || c.head_dim % 2 || c.rotary_dim % 2 || c.rotary_dim > c.head_dim ||
      c.layers > 128 || c.heads > 256 || c.head_dim > 512 || c.hidden > 16384 || c.intermediate > 131072 || c.vocab > 1000000)
    return fail(WGD_EINVAL, "Unsupported model dimensions.");
  if (c.family != 0 && c.family != 1) return fail(WGD_EINVAL, "family must be 0 (dense) or 1 (gemma3)");
  if (context_len < 1 || context_len > 32768) return fail(WGD_EINVAL, "Context must be an integer from 256 to 32768 tokens.");
  if (max_batch < 1 || max_batch > 128) return fail(WGD_EINVAL, "Batch size must be 1, 8, 16, 32, 64 or 128.");
  if (c.heads % ctx->tp_size || c.kv_heads % ctx->tp_size)
    return fail(WGD_EINVAL, "query and KV head counts must divide by the tensor-parallel size");
  if (c.heads / c.kv_heads > 8) return fail(WGD_EINVAL, "query heads per KV head above 8 are not supported");
  if (c.head_dim % 4) return fail(WGD_EINVAL, "head dimension must be a multiple of 4");
  ctx->c = c;
  ctx->context = context_len;
  ctx->max_batch = max_batch;
  ctx->begun = true;
  return WGD_OK;
}

int wgd_tensor_register(wgd_ctx *ctx, const char *name, int ggml_type, const uint64_t *dims, int nd, uint64_t file_offset,
                        uint64_t bytes, uint64_t row_bytes) {
  if (!ctx || !name || !dims) return fail(WGD_EINVAL, "null argument");
  if (!ctx->begun || ctx->ended) return fail(WGD_ESTATE, "tensor_register must come between model_begin and model_end");
  if (nd < 1 || nd > 4) return fail(WGD_EINVAL, "Invalid tensor directory.");
  if (ctx->by_name.count(name)) return fail(WGD_EINVAL, std::string("duplicate tensor ") + name);
  TensorRec t;
  t.name = name;
  t.type = ggml_type;
  t.nd = nd;
  uint64_t n = 1;
  for (int i = 0; i < nd; i++) { t.dims[i] = dims[i]; n *= dims[i]; }
  t.offset = file_offset;
  t.bytes = bytes;
  t.row_bytes = row_bytes;
  t.cols = (int64_t)dims[0];
  t.rows = (int64_t)(n / (dims[0] ? dims[0] : 1));
  if (type_supported(ggml_type)) {
    if (t.cols % block_elems(ggml_type) || (int64_t)row_bytes != gguf_row_bytes(ggml_type, t.cols) ||
        bytes != row_bytes * (uint64_t)t.rows)
      return fail(WGD_EINVAL, std::string("Invalid shape for ") + name + ".");
  }
  if (t.name == "token_embd.weight") t.role = R_EMBD;
  else if (t.name == "output_norm.weight") t.role = R_OUT_NORM;
  else if (t.name == "output.weight") t.role = R_OUTPUT;
  else {
    int layer; Role role;
    if (parse_layer_name(t.name, layer, role) && layer < ctx->c.layers) { t.layer = layer; t.role = role; }
  }
  ctx->by_name[t.name] = (int)ctx->tensors.size();
  ctx->tensors.push_back(t);
  return WGD_OK;
}

}  // extern "C"

static TensorRec *find(wgd_ctx *ctx, const std::string &name) {
  auto it = ctx->by_name.find(name);
  return it == ctx->by_name.end() ? nullptr : &ctx->tensors[it->second];
}

static int expect(wgd_ctx *ctx, const std::string &name, int64_t cols, int64_t rows, TensorRec **out, bool optional = false) {
  TensorRec *t = find(ctx, name);
  if (!t) {
    if (optional) { *out = nullptr; return WGD_OK; }
    return fail(WGD_EINVAL, "Missing or invalid tensor " + name + ".");
  }
  if (t->cols != cols || t->rows != rows || (rows == 1 && t->nd != 1))
    return fail(WGD_EINVAL, "Missing or invalid tensor " + name + ".");
  if (!type_supported(t->type))
    return fail(WGD_EINVAL, "Unsupported tensor quantization " + std::to_string(t->type) + " in " + name + ".");
  t->needed = true;
  *out = t;
  return WGD_OK;
}

static int alloc_linear(wgd_ctx *ctx, DevLinear &L, int type, int rows, int cols, const char *label) {
  L.type = type;
  L.rows = rows;
  L.cols = cols;
  L.nb = cols / block_elems(type);
  L.drow = dev_row_bytes(type, cols);
  L.tiled = tiled_type(type) && gemv2_max_batch(cols) > 0;
  if (cols % 32) return fail(WGD_EINVAL, std::string("matrix width must be a multiple of 32: ") + label);
  if (!L.tiled && gemv_max_batch(cols) == 0) return fail(WGD_EINVAL, std::string("matrix too wide for the GEMV kernel: ") + label);
  if (L.tiled) {
    const size_t pf = gemv2_part_floats(type, rows, cols, ctx->sm_count);
    if (pf > ctx->g2_part_floats) ctx->g2_part_floats = pf;
    if ((rows + 15) / 16 > ctx->g2_ctr_count) ctx->g2_ctr_count = (rows + 15) / 16;
    ctx->tc_cols_max = std::max(ctx->tc_cols_max, cols);  // tiled types (Q4_K, Q6_K) have a prompt-batch GEMM
    ctx->tc_rows_max = std::max(ctx->tc_rows_max, rows);
  }
  L.unit_rows = L.tiled ? TILE_ROWS : GEMV_ROWS;  // pages cut at whole tiles / whole gate|up interleave blocks
  L.label = label;
  ctx->pending.push_back(&L);  // storage is placed once every fixed buffer is (place_matrices)
  return WGD_OK;
}

// The residency rule, with no device calls: matrices of `sizes` device bytes (execution order)
// all stay on the device when they fit the budget beside `allocated`; otherwise two page slots of
// max(page, largest page unit) bytes are reserved first, and each matrix stays on the device only
// while it still fits with a 16 MiB margin (the cacheBudget rule of pager.ts:22), the rest streams.
// Returns whether anything streams; *slot_bytes is the slot size then (else 0).
static bool plan_residency(const uint64_t *sizes, int n, uint64_t allocated, uint64_t budget, uint64_t page_bytes,
                           uint64_t unit_max, int32_t *resident, uint64_t *slot_bytes) {
  const uint64_t margin = 16u << 20;
  uint64_t need = 0;
  for (int i = 0; i < n; i++) need += sizes[i];
  const bool paging = allocated + need > budget;
  *slot_bytes = 0;
  if (paging) {
    *slot_bytes = std::max(page_bytes, unit_max);
    allocated += 2 * (uint64_t)align_up((int64_t)*slot_bytes, 256);  // what ctx_alloc charges for the two slots
  }
  for (int i = 0; i < n; i++) {
    resident[i] = !paging || allocated + sizes[i] + margin <= budget;
    if (resident[i]) allocated += sizes[i];
  }
  return paging;
}

extern "C" int wgd_plan_residency(const uint64_t *sizes, int n, uint64_t allocated, uint64_t budget, uint64_t page_bytes,
                                  uint64_t unit_max, int32_t *resident, uint64_t *slot_bytes) {
  if ((!sizes || !resident) && n > 0) return fail(WGD_EINVAL, "null argument");
  if (!slot_bytes || n < 0) return fail(WGD_EINVAL, "bad argument");
  for (int i = 0; i < n; i++)
    if (sizes[i] % 256) return fail(WGD_EINVAL, "matrix sizes are whole 256-byte allocation units");
  plan_residency(sizes, n, allocated, budget, page_bytes, unit_max, resident, slot_bytes);
  return WGD_OK;
}

// Places the matrices in execution order by plan_residency: on the device, or in pinned host memory
// mapped into the device address space (repacked there at upload, copied page by page into the
// slots per forward).
static int place_matrices(wgd_ctx *ctx) {
  std::vector<uint64_t> sizes;
  int64_t unit_max = 0;
  for (DevLinear *L : ctx->pending) {
    sizes.push_back((uint64_t)align_up(L->bytes() + 16, 256));
    unit_max = std::max(unit_max, L->unit_bytes());
  }
  std::vector<int32_t> on_device(sizes.size());
  uint64_t slot_bytes = 0;
  ctx->paging = plan_residency(sizes.data(), (int)sizes.size(), ctx->allocated, ctx->budget, ctx->page_bytes,
                               (uint64_t)unit_max, on_device.data(), &slot_bytes);
  int rc;
  if (ctx->paging) {
    ctx->slot_bytes = (size_t)slot_bytes;
    for (int i = 0; i < 2; i++)
      if ((rc = ctx_alloc_t(ctx, &ctx->slot[i], ctx->slot_bytes, "page slot"))) return rc;
    CK(cudaStreamCreateWithFlags(&ctx->copy_stream, cudaStreamNonBlocking));
    for (int i = 0; i < 2; i++) {
      CK(cudaEventCreateWithFlags(&ctx->copied[i], cudaEventDisableTiming));
      CK(cudaEventCreateWithFlags(&ctx->freed[i], cudaEventDisableTiming));
      CK(cudaEventRecord(ctx->freed[i], ctx->stream));
    }
    ctx->st.page_bytes = ctx->slot_bytes;
  }
  uint64_t resident = 0;
  for (size_t i = 0; i < ctx->pending.size(); i++) {
    DevLinear *L = ctx->pending[i];
    const uint64_t size = sizes[i];
    if (on_device[i]) {
      if ((rc = ctx_alloc_t(ctx, &L->w, (size_t)size, L->label))) return rc;
      resident += size;
    } else {
      void *h = nullptr;
      cudaError_t e = cudaHostAlloc(&h, size, cudaHostAllocMapped | cudaHostAllocPortable);
      if (e != cudaSuccess) return fail(WGD_ECUDA, std::string("pinned host memory for a streamed matrix: ") + cudaGetErrorString(e));
      ctx->host_allocs.push_back(h);
      memset(h, 0, size);
      CK(cudaHostGetDevicePointer((void **)&L->w, h, 0));
      L->streamed = true;
    }
  }
  ctx->st.cache_bytes = resident;
  return WGD_OK;
}

// A matrix part: GGUF rows [src_begin, src_end) -> device rows (map), columns [blk0, blk0+nbl) in blocks.
static void place(TensorRec *t, DevLinear *L, int src_begin, int src_end, int dst_base, int interleave, int blk0, int nbl) {
  t->lin = L;
  t->map = RowMap{src_begin, src_end, dst_base, interleave, L->tiled ? TILE_ROWS / 2 : GEMV_ROWS / 2};
  t->blk0 = blk0;
  t->nbl = nbl;
}
static int place_vec(wgd_ctx *ctx, TensorRec *t, float *dst, int src0, int len) {
  if (!t) return WGD_OK;
  if (t->rows != 1) return fail(WGD_EINVAL, "vector tensor expected: " + t->name);
  t->vec = dst;
  t->vec_src0 = src0;
  t->vec_len = len;
  (void)ctx;
  return WGD_OK;
}

// The persistent decode plan: one PPhase per projection / attention of every layer,
// then the LM head. Built only for shapes the kernel covers; otherwise decode
// keeps the per-kernel path (persist_why says why).
static int build_persist_plan(wgd_ctx *ctx) {
  const wgd_model_config &c = ctx->c;
  const int H = c.hidden, hd = c.head_dim;
  ctx->persist_ok = false;
  auto no = [&](const char *why) { ctx->persist_why = why; return WGD_OK; };
  if (ctx->paging) return no("weights are paged through device slots (per-kernel path)");
  if (ctx->tp_size > P_TP_MAX) return no("more tensor-parallel ranks than the kernel's exchange holds");
  if (ctx->tp_size > 1 && ctx->sm_count + 1 > P_CAND_STRIDE) return no("more CTAs than the cross-rank candidate table holds");
  if (c.family == 1) return no("the gemma block (post-norms) uses the per-kernel path");
  const int G = ctx->kv_l ? ctx->heads_l / ctx->kv_l : 0;
  if (ctx->kv_l > ctx->sm_count) return no("more kv heads than CTAs (one attention item per CTA)");
  if (hd % 16 || hd > 128 || G < 1 || G > 8)
    return no("attention shape outside the persistent kernel (head_dim 16..128 in steps of 16, GQA group <= 8)");
  auto tiled_ok = [](const DevLinear &L) { return L.tiled && L.cols % 256 == 0 && L.cols >= 256; };
  if (!tiled_ok(ctx->lm)) return no("the LM head is not in the tiled layout");
  int max_cols = H;
  for (auto &L : ctx->layers) {
    if (!tiled_ok(L.qkv) || !tiled_ok(L.o) || !tiled_ok(L.gate_up) || !tiled_ok(L.down))
      return no("a projection is not in the tiled layout (Q4_K/Q6_K, width a multiple of 256)");
    max_cols = std::max(max_cols, std::max(L.o.cols, L.down.cols));
  }
  if (max_cols > 16384) return no("a projection input is wider than the kernel's digit records");
  const int tpn = ctx->tp_size;
  // tensor parallelism: the summed input row of a phase (hidden plus the peers' partials) sits in
  // shared memory behind that phase's digit records
  const int row_cols = tpn > 1 ? H : 0;
  int ns = persist_max_stages(max_cols, G, hd, row_cols);
  if (const char *v = getenv("WGD_PERSIST_STAGES")) ns = std::min(ns, std::max(3, atoi(v)));  // tuning override
  if (ns < 3) return no("not enough shared memory for the weight ring");
  int xs = 0;
  const size_t smem = persist_smem_bytes(max_cols, G, hd, ns, &xs, row_cols);
  const int grid = ctx->sm_count;
  const bool gemma = false, qkn = c.qk_norm != 0;
  std::vector<PPhase> plan;
  // residual stream: one buffer at tp = 1 (the O and down epilogues add into it); at tp > 1 two,
  // alternating between the phases that sum the ranks' partial rows (hb[1] = the projection buffer)
  float *hb[2] = {ctx->hidden, tpn > 1 ? ctx->proj : ctx->hidden};
  for (size_t li = 0; li < ctx->layers.size(); li++) {
    Layer &L = ctx->layers[li];
    auto gemv_phase = [&](const DevLinear &W, const float *x, const float *norm_w, float *y, const float *bias, int epi) {
      PPhase p{};
      p.kind = PH_GEMV;
      p.g.w = W.w;
      p.g.type = W.type;
      p.g.rows = W.rows;
      p.g.cols = W.cols;
      p.g.tiles = (W.rows + 15) / 16;
      p.g.nkb = W.cols / 256;
      p.g.x = x;
      p.g.norm_w = norm_w;
      p.g.eps = c.epsilon;
      p.g.y = y;
      p.g.bias = bias;
      p.g.epi = epi;
      return p;
    };
    {
      PPhase p = gemv_phase(L.qkv, tpn > 1 && li > 0 ? hb[1] : hb[0], L.attn_norm, ctx->qkv, L.qkv_bias, EPI_STORE);
      if (tpn > 1 && li > 0) {  // hb[1] + the ranks' down partials of the previous layer -> hb[0]
        p.g.xsum = 2;
        p.g.x_out = hb[0];
      }
      plan.push_back(p);
    }
    PPhase at{};
    at.kind = PH_ATTN;
    at.a.qkv = ctx->qkv;
    at.a.k = L.k_cache;
    at.a.v = L.v_cache;
    at.a.out = ctx->att;
    at.a.q_norm = L.q_norm;
    at.a.k_norm = L.k_norm;
    at.a.table = L.rope_table;
    at.a.heads = ctx->heads_l;
    at.a.kv_heads = ctx->kv_l;
    at.a.hd = hd;
    at.a.capacity = L.capacity;
    at.a.window = L.window;
    at.a.rot = gemma ? hd : (c.rotary_dim ? c.rotary_dim : hd);
    at.a.mode = qkn ? 0 : c.rope_mode;
    at.a.scale = c.attention_scale;
    at.a.eps = c.epsilon;
    plan.push_back(at);
    const int epi = !c.ffn_gate ? EPI_SILU : c.activation == 1 ? EPI_GLU_GELU : EPI_GLU_SILU;
    if (tpn == 1) {
      plan.push_back(gemv_phase(L.o, ctx->att, nullptr, ctx->hidden, L.o_bias, EPI_ADD));
      plan.push_back(gemv_phase(L.gate_up, ctx->hidden, L.ffn_norm, ctx->act, nullptr, epi));
      plan.push_back(gemv_phase(L.down, ctx->act, nullptr, ctx->hidden, nullptr, EPI_ADD));
    } else {
      PPhase o = gemv_phase(L.o, ctx->att, nullptr, nullptr, L.o_bias, EPI_STORE);
      o.g.push = 1;  // partial rows -> slot 0 of every rank
      plan.push_back(o);
      PPhase gu = gemv_phase(L.gate_up, hb[0], L.ffn_norm, ctx->act, nullptr, epi);
      gu.g.xsum = 1;  // hb[0] + the ranks' O partials -> hb[1]
      gu.g.x_out = hb[1];
      plan.push_back(gu);
      PPhase dn = gemv_phase(L.down, ctx->act, nullptr, nullptr, nullptr, EPI_STORE);
      dn.g.push = 2;  // partial rows -> slot 1 of every rank
      plan.push_back(dn);
    }
  }
  {
    PPhase p{};
    p.kind = PH_GEMV;
    p.g.w = ctx->lm.w;
    p.g.type = ctx->lm.type;
    p.g.rows = ctx->lm.rows;
    p.g.cols = H;
    p.g.tiles = (ctx->lm.rows + 15) / 16;
    p.g.nkb = H / 256;
    p.g.x = tpn > 1 ? hb[1] : ctx->hidden;
    if (tpn > 1) p.g.xsum = 2;  // + the ranks' down partials of the last layer
    p.g.norm_w = ctx->out_norm;
    p.g.eps = c.epsilon;
    p.g.y = ctx->logits;
    p.g.epi = EPI_STORE;
    p.g.argmax = 1;
    plan.push_back(p);
  }
  PersistArgs &a = ctx->pargs;
  a = PersistArgs{};
  PPhase *d_plan = nullptr;
  float *att_part = nullptr;
  unsigned *att_ctr = nullptr, *bar = nullptr;
  float2 *cand = nullptr;
  int *status = nullptr, rc;
  const int nsp_max = std::max(1, std::min(64, grid / ctx->kv_l));
  if ((rc = ctx_alloc(ctx, (void **)&d_plan, plan.size() * sizeof(PPhase), "decode plan")) ||
      (rc = ctx_alloc_t(ctx, &att_part, (size_t)ctx->kv_l * nsp_max * G * (hd + 4), "decode attention partials")) ||
      (rc = ctx_alloc_t(ctx, &att_ctr, (size_t)ctx->kv_l, "decode attention counters")) ||
      (rc = ctx_alloc_t(ctx, &cand, (size_t)grid, "decode candidates")) || (rc = ctx_alloc_t(ctx, &bar, 4, "grid barrier")) ||
      (rc = ctx_alloc_t(ctx, &status, 4, "decode status")))
    return rc;

  CK(cudaMemcpy(d_plan, plan.data(), plan.size() * sizeof(PPhase), cudaMemcpyHostToDevice));
  int *d_cancel = nullptr;
  CK(cudaHostGetDevicePointer((void **)&d_cancel, ctx->h_io + IO_CANCEL, 0));
  a.phases = d_plan;
  a.nphases = (int)plan.size();
  a.embd = ctx->embd.w;
  a.embd_type = ctx->embd.type;
  a.embd_tiled = ctx->embd.tiled ? 1 : 0;
  a.embd_drow = ctx->embd.drow;
  a.hidden = H;
  a.vocab = c.vocab;
  a.embd_scale = 1.f;
  a.x = ctx->hidden;
  a.tokens = ctx->d_tokens;
  a.cancel = d_cancel;
  a.att_part = att_part;
  a.att_ctr = att_ctr;
  a.cand = cand;
  a.bar = bar;
  a.status = status;
  a.nstage = ns;
  a.xs_bytes = xs;
  a.nsp_max = nsp_max;
  // four ring stages of the weight stream are also requested into L2 ahead of their shared-memory
  // copies (measured on the 8-layer model, 0 / 4 / 8 / 16 / 24 stages: 735 / 723 / 727 / 805 / 800 us
  // per token in one build, 660 / 653 for 0 / 4 in another; deeper look-ahead competes with the loads
  // of the latency-bound phases)
  a.l2_ahead = 4;
  a.tp = tpn;
  a.rank = ctx->tp_rank;
  a.vocab0 = ctx->vocab0;
  if (const char *v = getenv("WGD_PERSIST_L2_AHEAD")) a.l2_ahead = std::max(0, std::min(64, atoi(v)));  // tuning override
  (void)smem;
  ctx->persist_ok = true;
  ctx->persist_why = "";
  return WGD_OK;
}

// Runs `steps` greedy tokens from (first, start) in one launch; the tokens land in
// d_tokens and the status words in h_io[IO_STATUS..]. Stream-ordered (no sync).
// Per-launch state of the persistent kernel: the grid-barrier counter starts at zero; under tensor
// parallelism, the peers' exchange buffers and the cross-rank counter base of this launch.
static int persist_prepare(wgd_ctx *ctx, PersistArgs &a) {
  CK(cudaMemsetAsync(a.bar, 0, 3 * sizeof(unsigned), ctx->stream));  // the barrier counters grow from 0 within a launch
  if (ctx->tp_size > 1) {
    if (ctx->tp_broken)
      return fail(WGD_ETIMEOUT, "a tensor-parallel peer did not answer within the wait limit earlier; reload the model");
    TpPersistView v{};
    std::string err;
    if (tp_persist_view(ctx->tp, &v, &err)) return fail(WGD_ESTATE, err);
    for (int j = 0; j < P_TP_MAX; j++) a.xbuf[j] = v.buf[j];
    a.x_bar = v.bar;
    a.x_cand = v.cand;
    a.x_slot = v.slot;
    a.xbase = ctx->x_arrivals;
    a.xstep0 = ctx->x_tokens;
    a.x_limit_ns = ctx->tp_spin_limit ? ctx->tp_spin_limit * 1000ull : 2000000000ull;
  }
  return WGD_OK;
}

// After a persistent launch has completed: the cross-rank barriers it passed (two per layer and
// one per token), identical on every rank of the group, advance the counter base of the next.
static void persist_account(wgd_ctx *ctx) {
  if (ctx->tp_size < 2) return;
  const unsigned done = (unsigned)ctx->h_io[IO_STATUS + 1];
  if (ctx->h_io[IO_STATUS] == 1) ctx->tp_broken = true;
  ctx->x_arrivals += done * (2u * (unsigned)ctx->c.layers + 1u) * (unsigned)ctx->tp_size;
  ctx->x_tokens += done;
}

static int enqueue_persist(wgd_ctx *ctx, int first, int start, int steps) {
  PersistArgs a = ctx->pargs;
  a.first = first;
  a.start = start;
  a.steps = steps;
  int rc;
  CK(cudaMemsetAsync(a.status, 0, 4 * sizeof(int), ctx->stream));
  if ((rc = persist_prepare(ctx, a))) return rc;
  CK(launch_persist(a, ctx->sm_count, ctx->stream));
  CK(cudaMemcpyAsync(ctx->h_io + IO_STATUS, a.status, 4 * sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
  ctx->kernels = 1;
  ctx->st.kernel_launches += 1;
  return WGD_OK;
}

// Maps the persistent kernel's status word to the API's errors.
static int persist_status(wgd_ctx *ctx) {
  persist_account(ctx);
  switch (ctx->h_io[IO_STATUS]) {
    case 0: return WGD_OK;
    case 2: return fail(WGD_ENONFINITE, "Inference produced non-finite logits. Stop and report this model/runtime combination.");
    case 3: return fail(WGD_ECANCELLED, "Stopped by user");
    default: return fail(WGD_ETIMEOUT, "a wait inside the decode kernel ran past its limit");
  }
}

extern "C" int wgd_model_end(wgd_ctx *ctx) {
  if (!ctx) return fail(WGD_EINVAL, "null context");
  if (!ctx->begun || ctx->ended) return fail(WGD_ESTATE, "model_end out of order");
  CK(cudaSetDevice(ctx->device));
  const wgd_model_config &c = ctx->c;
  const int H = c.hidden, hd = c.head_dim, tp = ctx->tp_size, r = ctx->tp_rank;
  const bool gemma = c.family == 1;
  ctx->heads_l = c.heads / tp;
  ctx->kv_l = c.kv_heads / tp;
  ctx->q_l = ctx->heads_l * hd;
  ctx->kvd_l = ctx->kv_l * hd;
  ctx->qkv_rows = ctx->q_l + 2 * ctx->kvd_l;
  const int qd = c.heads * hd, kvd = c.kv_heads * hd;
  int rc;

  // ---- directory validation (modelConfig shape checks, gguf.ts:158-212)
  TensorRec *embd, *onorm, *output;
  if ((rc = expect(ctx, "token_embd.weight", H, c.vocab, &embd))) return rc;
  if ((rc = expect(ctx, "output_norm.weight", H, 1, &onorm))) return rc;
  if ((rc = expect(ctx, "output.weight", H, c.vocab, &output, true))) return rc;
  ctx->tied = output == nullptr;
  // FFN partition unit: the down projection's block width (row-split by columns).
  TensorRec *down0 = find(ctx, "blk.0.ffn_down.weight");
  if (!down0 || !type_supported(down0->type)) return fail(WGD_EINVAL, "Missing or invalid tensor blk.0.ffn_down.weight.");
  const int funit = block_elems(down0->type);
  if (c.intermediate % funit) return fail(WGD_EINVAL, "feed-forward width is not a whole number of blocks");
  const int fblocks = c.intermediate / funit;
  ctx->ffn0 = part_begin(fblocks, r, tp) * funit;
  ctx->ffn_l = part_begin(fblocks, r + 1, tp) * funit - ctx->ffn0;
  if (ctx->ffn_l % 2) return fail(WGD_EINVAL, "feed-forward shard must have an even row count");
  // vocabulary rows split in whole 16-row tiles
  const int vt = (c.vocab + 15) / 16;
  ctx->vocab0 = std::min(c.vocab, part_begin(vt, r, tp) * 16);
  ctx->vocab_l = std::min(c.vocab, part_begin(vt, r + 1, tp) * 16) - ctx->vocab0;

  ctx->layers.assign(c.layers, Layer());
  const int B = ctx->max_batch;
  for (int l = 0; l < c.layers; l++) {
    Layer &L = ctx->layers[l];
    const std::string p = "blk." + std::to_string(l) + ".";
    TensorRec *an, *q, *k, *v, *o, *qb = nullptr, *kb = nullptr, *vb = nullptr, *ob = nullptr, *qn = nullptr, *kn = nullptr;
    TensorRec *pa = nullptr, *fn, *gate = nullptr, *up, *dn, *pf = nullptr;
    if ((rc = expect(ctx, p + "attn_norm.weight", H, 1, &an))) return rc;
    if ((rc = expect(ctx, p + "attn_q.weight", H, qd, &q))) return rc;
    if ((rc = expect(ctx, p + "attn_k.weight", H, kvd, &k))) return rc;
    if ((rc = expect(ctx, p + "attn_v.weight", H, kvd, &v))) return rc;
    if ((rc = expect(ctx, p + "attn_output.weight", qd, H, &o))) return rc;
    if ((rc = expect(ctx, p + "ffn_norm.weight", H, 1, &fn))) return rc;
    if ((rc = expect(ctx, p + "ffn_up.weight", H, c.intermediate, &up))) return rc;
    if ((rc = expect(ctx, p + "ffn_down.weight", c.intermediate, H, &dn))) return rc;
    const bool gated = gemma || c.ffn_gate;
    if (gated && (rc = expect(ctx, p + "ffn_gate.weight", H, c.intermediate, &gate))) return rc;
    if (!gemma) {
      if (c.bias_q && (rc = expect(ctx, p + "attn_q.bias", qd, 1, &qb))) return rc;
      if (c.bias_k && (rc = expect(ctx, p + "attn_k.bias", kvd, 1, &kb))) return rc;
      if (c.bias_v && (rc = expect(ctx, p + "attn_v.bias", kvd, 1, &vb))) return rc;
      if (c.bias_output && (rc = expect(ctx, p + "attn_output.bias", H, 1, &ob))) return rc;
    } else {
      if ((rc = expect(ctx, p + "post_attention_norm.weight", H, 1, &pa))) return rc;
      if ((rc = expect(ctx, p + "post_ffw_norm.weight", H, 1, &pf))) return rc;
    }
    if (gemma || c.qk_norm) {
      if ((rc = expect(ctx, p + "attn_q_norm.weight", hd, 1, &qn))) return rc;
      if ((rc = expect(ctx, p + "attn_k_norm.weight", hd, 1, &kn))) return rc;
    }
    if (q->type != k->type || q->type != v->type)
      return fail(WGD_EINVAL, "Q/K/V of one layer must share a quantization type (fused projection)");
    if (gate && gate->type != up->type)
      return fail(WGD_EINVAL, "ffn_gate and ffn_up of one layer must share a quantization type (fused projection)");
    if (dn->type != down0->type) return fail(WGD_EINVAL, "ffn_down must use one quantization type in every layer");
    if (ctx->q_l % block_elems(o->type) || (r * ctx->q_l) % block_elems(o->type))
      return fail(WGD_EINVAL, "attention output shard is not a whole number of blocks");

    // ---- placement: this rank's heads and FFN rows
    if ((rc = alloc_linear(ctx, L.qkv, q->type, ctx->qkv_rows, H, "qkv"))) return rc;
    place(q, &L.qkv, r * ctx->q_l, (r + 1) * ctx->q_l, 0, 0, 0, L.qkv.nb);
    place(k, &L.qkv, r * ctx->kvd_l, (r + 1) * ctx->kvd_l, ctx->q_l, 0, 0, L.qkv.nb);
    place(v, &L.qkv, r * ctx->kvd_l, (r + 1) * ctx->kvd_l, ctx->q_l + ctx->kvd_l, 0, 0, L.qkv.nb);
    if ((rc = alloc_linear(ctx, L.o, o->type, H, ctx->q_l, "attn_output"))) return rc;
    const int ob_ = block_elems(o->type);
    place(o, &L.o, 0, H, 0, 0, r * ctx->q_l / ob_, ctx->q_l / ob_);
    if (gated) {
      if ((rc = alloc_linear(ctx, L.gate_up, up->type, 2 * ctx->ffn_l, H, "ffn_gate_up"))) return rc;
      place(gate, &L.gate_up, ctx->ffn0, ctx->ffn0 + ctx->ffn_l, 0, 1, 0, L.gate_up.nb);
      place(up, &L.gate_up, ctx->ffn0, ctx->ffn0 + ctx->ffn_l, 0, 2, 0, L.gate_up.nb);
    } else {
      if ((rc = alloc_linear(ctx, L.gate_up, up->type, ctx->ffn_l, H, "ffn_up"))) return rc;
      place(up, &L.gate_up, ctx->ffn0, ctx->ffn0 + ctx->ffn_l, 0, 0, 0, L.gate_up.nb);
    }
    if ((rc = alloc_linear(ctx, L.down, dn->type, H, ctx->ffn_l, "ffn_down"))) return rc;
    place(dn, &L.down, 0, H, 0, 0, ctx->ffn0 / funit, ctx->ffn_l / funit);

    // ---- vectors
    if ((rc = ctx_alloc_t(ctx, &L.attn_norm, H, "attn_norm"))) return rc;
    place_vec(ctx, an, L.attn_norm, 0, H);
    if ((rc = ctx_alloc_t(ctx, &L.ffn_norm, H, "ffn_norm"))) return rc;
    place_vec(ctx, fn, L.ffn_norm, 0, H);
    if (qb || kb || vb) {
      if ((rc = ctx_alloc_t(ctx, &L.qkv_bias, ctx->qkv_rows, "qkv_bias"))) return rc;
      place_vec(ctx, qb, L.qkv_bias, r * ctx->q_l, ctx->q_l);
      place_vec(ctx, kb, L.qkv_bias + ctx->q_l, r * ctx->kvd_l, ctx->kvd_l);
      place_vec(ctx, vb, L.qkv_bias + ctx->q_l + ctx->kvd_l, r * ctx->kvd_l, ctx->kvd_l);
    }
    if (ob && r == 0) {  // the output bias is added once across the tensor-parallel sum
      if ((rc = ctx_alloc_t(ctx, &L.o_bias, H, "o_bias"))) return rc;
      place_vec(ctx, ob, L.o_bias, 0, H);
    } else if (ob) {
      ob->needed = false;
    }
    if (qn) {
      if ((rc = ctx_alloc_t(ctx, &L.q_norm, hd, "q_norm")) || (rc = ctx_alloc_t(ctx, &L.k_norm, hd, "k_norm"))) return rc;
      place_vec(ctx, qn, L.q_norm, 0, hd);
      place_vec(ctx, kn, L.k_norm, 0, hd);
    }
    if (pa) {
      if ((rc = ctx_alloc_t(ctx, &L.post_attn, H, "post_attention_norm")) || (rc = ctx_alloc_t(ctx, &L.post_ffw, H, "post_ffw_norm")))
        return rc;
      place_vec(ctx, pa, L.post_attn, 0, H);
      place_vec(ctx, pf, L.post_ffw, 0, H);
    }
    // ---- attention window and KV ring capacity (context.ts:16-24; engine.ts:147,161,163,234)
    L.local = gemma && c.period > 1 && l % c.period != c.period - 1;
    L.theta = L.local ? c.local_theta : c.theta;
    L.rope_scale = L.local ? 1.0 : c.rope_scale;
    if (gemma) {
      L.window = L.local ? c.window : ctx->context;
      L.capacity = L.local ? std::min(ctx->context, c.window + B - 1) : ctx->context;
    } else {
      L.window = c.sliding_window > 0 ? c.sliding_window : ctx->context;
      L.capacity = c.sliding_window > 0 ? std::min(ctx->context, c.sliding_window + B - 1) : ctx->context;
    }
    if ((rc = ctx_alloc_t(ctx, &L.k_cache, (size_t)ctx->kv_l * L.capacity * hd, "K cache"))) return rc;
    if ((rc = ctx_alloc_t(ctx, &L.v_cache, (size_t)ctx->kv_l * L.capacity * hd, "V cache"))) return rc;
  }

  // ---- embedding (replicated: any id can appear) and LM head (vocab rows of this rank)
  // the head is used every token, the embedding table one row per token: place the head first
  if (!ctx->tied) {
    if ((rc = alloc_linear(ctx, ctx->lm, output->type, ctx->vocab_l, H, "output"))) return rc;
    place(output, &ctx->lm, ctx->vocab0, ctx->vocab0 + ctx->vocab_l, 0, 0, 0, ctx->lm.nb);
  }
  if ((rc = alloc_linear(ctx, ctx->embd, embd->type, c.vocab, H, "token_embd"))) return rc;
  place(embd, &ctx->embd, 0, c.vocab, 0, 0, 0, ctx->embd.nb);
  if ((rc = ctx_alloc_t(ctx, &ctx->out_norm, H, "output_norm"))) return rc;
  place_vec(ctx, onorm, ctx->out_norm, 0, H);

  // ---- work buffers
  const int F = std::max(ctx->ffn_l, 1);
  if ((rc = ctx_alloc_t(ctx, &ctx->hidden, (size_t)B * H, "hidden")) || (rc = ctx_alloc_t(ctx, &ctx->qkv, (size_t)B * ctx->qkv_rows, "qkv")) ||
      (rc = ctx_alloc_t(ctx, &ctx->qrot, (size_t)B * ctx->q_l, "q")) || (rc = ctx_alloc_t(ctx, &ctx->att, (size_t)B * ctx->q_l, "attention")) ||
      (rc = ctx_alloc_t(ctx, &ctx->proj, (size_t)B * H, "projection")) || (rc = ctx_alloc_t(ctx, &ctx->act, (size_t)B * F, "ffn")) ||
      (rc = ctx_alloc_t(ctx, &ctx->logits, (size_t)c.vocab, "logits")) || (rc = ctx_alloc_t(ctx, &ctx->d_ids, (size_t)B, "ids")) ||
      (rc = ctx_alloc_t(ctx, &ctx->d_start, 4, "start")) || (rc = ctx_alloc_t(ctx, &ctx->d_argmax, 4, "argmax")) ||
      (rc = ctx_alloc_t(ctx, &ctx->d_err, 4, "err")) || (rc = ctx_alloc_t(ctx, &ctx->d_maxval, 4, "maxval")) ||
      (rc = ctx_alloc_t(ctx, &ctx->d_tokens, (size_t)ctx->context, "decoded tokens")) || (rc = ctx_alloc_t(ctx, &ctx->d_step, 4, "step")))
    return rc;
  ctx->att_splits = attention_splits(ctx->context);
  if ((rc = ctx_alloc_t(ctx, &ctx->att_part, attention_part_floats(B, c.heads / tp, ctx->kv_l, hd, ctx->att_splits), "attention partials")))
    return rc;
  if ((rc = ctx_alloc_t(ctx, &ctx->att_ctr, (size_t)B * ctx->kv_l, "attention counters"))) return rc;
  if ((rc = ctx_alloc_t(ctx, &ctx->am_part, 2 * 256, "argmax partials")) || (rc = ctx_alloc_t(ctx, &ctx->am_ctr, 4, "argmax counter")))
    return rc;
  if ((rc = ctx_alloc_t(ctx, &ctx->d_sparams, 1, "sampling settings")) ||
      (rc = ctx_alloc_t(ctx, &ctx->d_uniform, (size_t)ctx->context, "sampling draws")) ||
      (rc = ctx_alloc_t(ctx, &ctx->smp_part, (size_t)SAMPLE_MAX_GRID * SAMPLE_MAX_K, "sampling candidates")) ||
      (rc = ctx_alloc_t(ctx, &ctx->smp_ctr, 4, "sampling counter")) || (rc = ctx_alloc_t(ctx, &ctx->d_ptok, 4, "decode token slot")))
    return rc;
  ctx->staging_bytes = 64u << 20;
  if ((rc = ctx_alloc_t(ctx, &ctx->staging, ctx->staging_bytes, "upload staging"))) return rc;
  // RoPE (cos, sin) tables, one per distinct (theta, scale): angle = pos * scale / theta^(2i/rot),
  // evaluated in double and rounded once to float (the rope kernels read them)
  {
    const int rot = gemma ? hd : (c.rotary_dim ? c.rotary_dim : hd), half = rot / 2;
    std::vector<float2> host((size_t)ctx->context * half);
    for (auto &L : ctx->layers) {
      const auto key = std::make_pair(L.theta, L.rope_scale);
      const float2 *found = nullptr;
      for (auto &kv : ctx->rope_tables)
        if (kv.first == key) found = kv.second;
      if (!found) {
        float2 *dev = nullptr;
        if ((rc = ctx_alloc_t(ctx, &dev, host.size(), "rope table"))) return rc;
        for (int pos = 0; pos < ctx->context; pos++)
          for (int i = 0; i < half; i++) {
            const double angle = (double)pos * L.rope_scale / std::pow(L.theta, (2.0 * i) / rot);
            host[(size_t)pos * half + i] = make_float2((float)std::cos(angle), (float)std::sin(angle));
          }
        CK(cudaMemcpy(dev, host.data(), host.size() * sizeof(float2), cudaMemcpyHostToDevice));
        ctx->rope_tables.push_back({key, dev});
        found = dev;
      }
      L.rope_table = found;
    }
  }
  if (ctx->g2_part_floats && ((rc = ctx_alloc_t(ctx, &ctx->g2_part, ctx->g2_part_floats, "gemv partials")) ||
                              (rc = ctx_alloc_t(ctx, &ctx->g2_ctr, (size_t)ctx->g2_ctr_count, "gemv tile counters"))))
    return rc;
  if (ctx->tc_cols_max && B >= 8) {
    if ((rc = ctx_alloc_t(ctx, &ctx->tc_panel, gemm_tc_panel_bytes(B, ctx->tc_cols_max), "GEMM activation panel")) ||
        (rc = ctx_alloc_t(ctx, &ctx->tc_part, gemm_tc_part_floats(B, ctx->sm_count), "GEMM partials")) ||
        (rc = ctx_alloc_t(ctx, &ctx->tc_ctr, (size_t)gemm_tc_mtiles(ctx->tc_rows_max), "GEMM counters")))
      return rc;
    CK(cudaHostGetDevicePointer((void **)&ctx->tc_status, ctx->h_io + IO_TC, 0));
  }
  if (tp > 1) {
    if ((rc = tp_create(&ctx->tp, ctx->tp_rank, tp, (size_t)B * H, &g_err))) return rc;
  }
  if ((rc = place_matrices(ctx))) return rc;
  if (ctx->tied) {  // the head is this rank's vocabulary rows of the embedding table
    ctx->lm = ctx->embd;
    ctx->lm.w = ctx->embd.w + (ctx->embd.tiled ? (int64_t)(ctx->vocab0 / 16) * ctx->embd.nb * tile_chunk_bytes(embd->type)
                                               : (int64_t)ctx->vocab0 * ctx->embd.drow);
    ctx->lm.rows = ctx->vocab_l;
  }
  if ((rc = build_persist_plan(ctx))) return rc;
  ctx->ended = true;
  ctx->st.gpu_bytes = ctx->allocated;
  ctx->st.peak_gpu_bytes = ctx->peak;
  return WGD_OK;
}

// ------------------------------------------------------------------ uploads

static int upload_vector(wgd_ctx *ctx, TensorRec *t, const void *host) {
  const int64_t n = t->cols;
  const int64_t drb = dev_row_bytes(t->type, n);
  const size_t need = (size_t)t->bytes + (size_t)drb + (size_t)n * 4 + 64;
  if (need > ctx->staging_bytes) return fail(WGD_EINVAL, "vector too large for staging: " + t->name);
  uint8_t *raw = ctx->staging, *packed = ctx->staging + align_up((int64_t)t->bytes, 256);
  float *vals = (float *)(packed + align_up(drb, 256));
  CK(cudaMemcpyAsync(raw, host, t->bytes, cudaMemcpyHostToDevice, ctx->stream));
  RowMap m{0, 1, 0, 0, 0};
  CK(launch_repack(t->type, raw, (int64_t)t->row_bytes, 0, 1, 0, (int)(n / block_elems(t->type)), packed, drb, m, ctx->stream));
  CK(launch_dequant(t->type, packed, drb, 1, (int)n, vals, n, ctx->stream));
  CK(cudaMemcpyAsync(t->vec, vals + t->vec_src0, sizeof(float) * t->vec_len, cudaMemcpyDeviceToDevice, ctx->stream));
  CK(cudaStreamSynchronize(ctx->stream));
  t->uploaded_rows = 1;
  return WGD_OK;
}

extern "C" int wgd_tensor_upload(wgd_ctx *ctx, const char *name, uint64_t byte_off, const void *host, uint64_t n) {
  if (!ctx || !name || !host) return fail(WGD_EINVAL, "null argument");
  if (!ctx->ended) return fail(WGD_ESTATE, "tensor_upload requires model_end first");
  CK(cudaSetDevice(ctx->device));
  TensorRec *t = find(ctx, name);
  if (!t) return fail(WGD_EINVAL, std::string("unknown tensor ") + name);
  if (!t->needed) return WGD_OK;  // not used by this rank / model
  if (t->vec) {
    if (byte_off != 0 || n != t->bytes) return fail(WGD_EINVAL, "vectors upload whole: " + t->name);
    return upload_vector(ctx, t, host);
  }
  if (!t->lin) return WGD_OK;
  if (byte_off % t->row_bytes || n % t->row_bytes || byte_off + n > t->bytes)
    return fail(WGD_EINVAL, "uploads must cover whole rows inside the tensor: " + t->name);
  int64_t row0 = (int64_t)(byte_off / t->row_bytes), nrows = (int64_t)(n / t->row_bytes);
  // clip to the rows this rank keeps
  int64_t keep0 = std::max<int64_t>(row0, t->map.src_begin), keep1 = std::min<int64_t>(row0 + nrows, t->map.src_end);
  const int64_t chunk_rows = std::max<int64_t>(1, (int64_t)ctx->staging_bytes / (int64_t)t->row_bytes);
  for (int64_t a = keep0; a < keep1; a += chunk_rows) {
    const int64_t cnt = std::min(chunk_rows, keep1 - a);
    const uint8_t *src = (const uint8_t *)host + (a - row0) * t->row_bytes;
    CK(cudaMemcpyAsync(ctx->staging, src, cnt * t->row_bytes, cudaMemcpyHostToDevice, ctx->stream));
    if (t->lin->tiled)
      CK(launch_repack_tiled(t->type, ctx->staging, (int64_t)t->row_bytes, (int)a, (int)cnt, t->blk0, t->nbl, t->lin->w,
                             t->lin->rows, t->map, ctx->stream));
    else
      CK(launch_repack(t->type, ctx->staging, (int64_t)t->row_bytes, (int)a, (int)cnt, t->blk0, t->nbl, t->lin->w, t->lin->drow,
                       t->map, ctx->stream));
    CK(cudaStreamSynchronize(ctx->stream));
  }
  t->uploaded_rows += nrows;
  ctx->st.uploads++;
  ctx->st.read_bytes += n;
  return WGD_OK;
}

extern "C" int wgd_tensor_host(wgd_ctx *ctx, const char *name, const void *host, int pinned) {
  if (!ctx || !name || !host) return fail(WGD_EINVAL, "null argument");
  TensorRec *t = find(ctx, name);
  if (!t) return fail(WGD_EINVAL, std::string("unknown tensor ") + name);
  (void)pinned;  // the staging copy below reads pageable and page-locked memory alike
  return wgd_tensor_upload(ctx, name, 0, host, t->bytes);
}

extern "C" int wgd_set_page_reader(wgd_ctx *ctx, wgd_read_fn fn, void *user) {
  if (!ctx) return fail(WGD_EINVAL, "null context");
  ctx->reader = fn;
  ctx->reader_user = user;
  return WGD_OK;
}

extern "C" int wgd_load_weights(wgd_ctx *ctx) {
  if (!ctx) return fail(WGD_EINVAL, "null context");
  if (!ctx->ended) return fail(WGD_ESTATE, "load_weights requires model_end first");
  if (!ctx->reader) return fail(WGD_ESTATE, "no page reader set (wgd_set_page_reader)");
  const uint64_t page = std::max<uint64_t>(ctx->page_bytes, 1u << 20);
  if (!ctx->reader_buf || ctx->reader_buf_bytes < page) {
    if (ctx->reader_buf) cudaFreeHost(ctx->reader_buf);
    ctx->reader_buf = nullptr;
    CK(cudaMallocHost((void **)&ctx->reader_buf, page));
    ctx->reader_buf_bytes = page;
  }
  for (auto &t : ctx->tensors) {
    if (!t.needed || (t.vec ? t.uploaded_rows >= 1 : t.uploaded_rows >= t.rows)) continue;
    // whole rows per read; a vector (or a row wider than a page) is read whole
    const uint64_t step = t.vec || t.row_bytes > page ? t.bytes : page / t.row_bytes * t.row_bytes;
    if (step > ctx->reader_buf_bytes) {
      cudaFreeHost(ctx->reader_buf);
      ctx->reader_buf = nullptr;
      CK(cudaMallocHost((void **)&ctx->reader_buf, step));
      ctx->reader_buf_bytes = step;
    }
    for (uint64_t off = 0; off < t.bytes; off += step) {
      const uint64_t n = std::min(step, t.bytes - off);
      const auto r0 = std::chrono::steady_clock::now();
      if (ctx->reader(ctx->reader_user, t.offset + off, n, ctx->reader_buf) != 0)
        return fail(WGD_EIO, "page reader failed for " + t.name);
      ctx->st.read_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - r0).count();
      int rc;
      if ((rc = wgd_tensor_upload(ctx, t.name.c_str(), off, ctx->reader_buf, n))) return rc;
    }
  }
  return WGD_OK;
}

static bool all_uploaded(wgd_ctx *ctx, std::string *missing) {
  for (auto &t : ctx->tensors) {
    if (!t.needed) continue;
    bool ok = t.vec ? t.uploaded_rows >= 1 : t.uploaded_rows >= t.rows;
    if (!ok) { if (missing) *missing = t.name; return false; }
  }
  return true;
}

extern "C" int wgd_model_ready(wgd_ctx *ctx, int *ready) {
  if (!ctx || !ready) return fail(WGD_EINVAL, "null argument");
  *ready = ctx->ended && all_uploaded(ctx, nullptr);
  return WGD_OK;
}

extern "C" int wgd_model_placement(wgd_ctx *ctx, uint64_t *resident, uint64_t *streamed) {
  if (!ctx) return fail(WGD_EINVAL, "null context");
  uint64_t res = 0;
  for (auto &L : ctx->layers) res += L.qkv.bytes() + L.o.bytes() + L.gate_up.bytes() + L.down.bytes();
  res += ctx->embd.bytes() + (ctx->tied ? 0 : ctx->lm.bytes());
  if (resident) *resident = res;
  if (streamed) *streamed = 0;
  return WGD_OK;
}

// ------------------------------------------------------------------ forward

static int gemv(wgd_ctx *ctx, const DevLinear &L, const float *x, int ldx, const float *norm_w, float *y, int ldy,
                const float *bias, int epi, int batch);

// A streamed matrix, one page at a time: the copy stream fills slot i (after the GEMV that last
// read it finished: event freed[i]) from pinned host memory, the compute stream waits for the copy
// (copied[i]) and runs the GEMV on that page's rows (WeightPager.page, pager.ts:25-44; the copy of
// the next page overlaps the GEMV of this one).
static int gemv_paged(wgd_ctx *ctx, const DevLinear &L, const float *x, int ldx, const float *norm_w, float *y, int ldy,
                      const float *bias, int epi, int batch) {
  const bool glu = epi == EPI_GLU_SILU || epi == EPI_GLU_GELU;
  const int64_t ub = L.unit_bytes();
  const int units = (L.rows + L.unit_rows - 1) / L.unit_rows;
  const int per_page = (int)std::max<int64_t>(1, (int64_t)ctx->slot_bytes / ub);
  const uint8_t *host = L.w;  // mapped host pointer: the same address from the host
  for (int u0 = 0; u0 < units; u0 += per_page) {
    const int n = std::min(per_page, units - u0);
    const int r0 = u0 * L.unit_rows, rows = std::min(n * L.unit_rows, L.rows - r0);
    const int i = (int)(ctx->page_seq++ & 1u);
    CK(cudaStreamWaitEvent(ctx->copy_stream, ctx->freed[i], 0));
    CK(cudaMemcpyAsync(ctx->slot[i], host + (int64_t)u0 * ub, (size_t)n * ub, cudaMemcpyHostToDevice, ctx->copy_stream));
    CK(cudaEventRecord(ctx->copied[i], ctx->copy_stream));
    CK(cudaStreamWaitEvent(ctx->stream, ctx->copied[i], 0));
    DevLinear P = L;
    P.streamed = false;
    P.w = ctx->slot[i];
    P.rows = rows;
    int rc;
    if ((rc = gemv(ctx, P, x, ldx, norm_w, y + (glu ? r0 / 2 : r0), ldy, bias ? bias + r0 : nullptr, epi, batch))) return rc;
    CK(cudaEventRecord(ctx->freed[i], ctx->stream));
    ctx->st.streamed_bytes += (uint64_t)n * ub;
  }
  return WGD_OK;
}

static int gemv(wgd_ctx *ctx, const DevLinear &L, const float *x, int ldx, const float *norm_w, float *y, int ldy,
                const float *bias, int epi, int batch) {
  if (L.streamed) return gemv_paged(ctx, L, x, ldx, norm_w, y, ldy, bias, epi, batch);
  if (L.tiled && ctx->tc_panel && ctx->tc_min_batch > 0 && batch >= ctx->tc_min_batch &&
      gemm_tc_supported(L.type, L.rows, L.cols, batch)) {
    GemmTcLaunch g{};
    g.type = L.type;
    g.w = L.w;
    g.rows = L.rows;
    g.cols = L.cols;
    g.x = x;
    g.ldx = ldx;
    g.norm_w = norm_w;
    g.eps = ctx->c.epsilon;
    g.y = y;
    g.ldy = ldy;
    g.bias = bias;
    g.epi = epi;
    g.batch = batch;
    g.panel = ctx->tc_panel;
    g.part = ctx->tc_part;
    g.ctr = ctx->tc_ctr;
    g.status = ctx->tc_status;
    ctx->kernels += 2;  // activation panel + GEMM
    CK(launch_gemm_tc(g, ctx->stream, ctx->sm_count));
    return WGD_OK;
  }
  const int chunk = L.tiled ? gemv2_max_batch(L.cols) : gemv_max_batch(L.cols);
  ctx->kernels += chunk > 0 ? (batch + chunk - 1) / chunk : 1;
  if (L.tiled) {
    Gemv2Launch g{};
    g.w = L.w;
    g.rows = L.rows;
    g.cols = L.cols;
    g.x = x;
    g.ldx = ldx;
    g.norm_w = norm_w;
    g.eps = ctx->c.epsilon;
    g.y = y;
    g.ldy = ldy;
    g.bias = bias;
    g.epi = epi;
    g.batch = batch;
    g.part = ctx->g2_part;
    g.part_floats = ctx->g2_part_floats;
    g.tile_ctr = ctx->g2_ctr;
    g.ctr_count = ctx->g2_ctr_count;
    CK(launch_gemv2(L.type, g, ctx->stream, true, ctx->sm_count));
    return WGD_OK;
  }
  GemvArgs a{};
  a.w = L.w;
  a.drow = L.drow;
  a.rows = L.rows;
  a.cols = L.cols;
  a.nb = L.nb;
  a.x = x;
  a.ldx = ldx;
  a.norm_w = norm_w;
  a.eps = ctx->c.epsilon;
  a.y = y;
  a.ldy = ldy;
  a.bias = bias;
  a.epi = epi;
  a.batch = batch;
  CK(launch_gemv(L.type, a, ctx->stream, true, ctx->sm_count));
  return WGD_OK;
}

// Sum of this rank's partial [n][H] into `hidden` across the tensor-parallel group.
static int tp_reduce_add(wgd_ctx *ctx, const float *partial, float *hidden, int n) {
  if (ctx->tp_size == 1) { CK(launch_add(partial, hidden, (int64_t)n * ctx->c.hidden, ctx->stream, true)); return WGD_OK; }
  return tp_allreduce_add(ctx->tp, partial, hidden, (size_t)n * ctx->c.hidden, ctx->stream, ctx->tp_spin_limit, &g_err);
}

// Enqueues one forward of n rows (positions from *d_start) on ctx->stream.
// io: copy ids/start in from pinned host memory and the argmax out again.
static int enqueue_forward(wgd_ctx *ctx, int n, bool want_logits_rows, bool io = true) {
  const wgd_model_config &c = ctx->c;
  const int H = c.hidden, hd = c.head_dim;
  const bool gemma = c.family == 1, tp1 = ctx->tp_size == 1;
  int rc;
  ctx->kernels = 0;
  if (io) {
    CK(cudaMemcpyAsync(ctx->d_start, ctx->h_io, sizeof(int32_t), cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(ctx->d_ids, ctx->h_io + 2, sizeof(int32_t) * n, cudaMemcpyHostToDevice, ctx->stream));
  }
  ctx->kernels += 1 + c.layers * 1 + 1 + (gemma ? 2 * c.layers : 0) + (tp1 ? 0 : 2 * c.layers + 1);
  CK(launch_embed(ctx->embd.type, ctx->embd.w, ctx->embd.drow, H, ctx->d_ids, n, c.vocab, gemma ? sqrtf((float)H) : 1.f,
                  ctx->hidden, H, ctx->d_err, ctx->stream, false, ctx->embd.tiled));
  for (int l = 0; l < c.layers; l++) {
    Layer &L = ctx->layers[l];
    if ((rc = gemv(ctx, L.qkv, ctx->hidden, H, L.attn_norm, ctx->qkv, ctx->qkv_rows, L.qkv_bias, EPI_STORE, n))) return rc;
    RopeArgs ra{};
    ra.qkv = ctx->qkv;
    ra.ld = ctx->qkv_rows;
    ra.n = n;
    ra.heads = ctx->heads_l;
    ra.kv_heads = ctx->kv_l;
    ra.hd = hd;
    const bool qkn = gemma || c.qk_norm;
    ra.rot = gemma ? hd : (c.rotary_dim ? c.rotary_dim : hd);
    ra.mode = qkn ? 0 : c.rope_mode;
    ra.q_norm = L.q_norm;
    ra.k_norm = L.k_norm;
    ra.eps = c.epsilon;
    ra.theta = L.theta;
    ra.scale = L.rope_scale;
    ra.table = L.rope_table;
    ra.start = ctx->d_start;
    ra.k_cache = L.k_cache;
    ra.v_cache = L.v_cache;
    ra.capacity = L.capacity;
    ra.q_out = ctx->qrot;
    const bool fuse_rope = n == 1;  // decode: the attention kernel rotates and writes the new K/V itself
    if (!fuse_rope) {
      CK(launch_rope_kv(ra, ctx->stream, true));
      ctx->kernels += 1;
    }
    AttnArgs aa{};
    aa.q = ctx->qrot;
    aa.k = L.k_cache;
    aa.v = L.v_cache;
    aa.out = ctx->att;
    aa.n = n;
    aa.heads = ctx->heads_l;
    aa.kv_heads = ctx->kv_l;
    aa.hd = hd;
    aa.capacity = L.capacity;
    aa.window = L.window;
    aa.scale = c.attention_scale;
    aa.start = ctx->d_start;
    aa.part = ctx->att_part;
    aa.ctr = ctx->att_ctr;
    aa.splits = ctx->att_splits;
    if (fuse_rope) {
      aa.qkv = ctx->qkv;
      aa.q_norm = L.q_norm;
      aa.k_norm = L.k_norm;
      aa.eps = c.epsilon;
      aa.rot = ra.rot;
      aa.mode = ra.mode;
      aa.table = L.rope_table;
    }
    CK(launch_attention(aa, ctx->stream, true));
    if (gemma) {
      if ((rc = gemv(ctx, L.o, ctx->att, ctx->q_l, nullptr, ctx->proj, H, nullptr, EPI_STORE, n))) return rc;
      if (!tp1 && (rc = tp_allreduce_inplace(ctx->tp, ctx->proj, (size_t)n * H, ctx->stream, ctx->tp_spin_limit, &g_err))) return rc;
      CK(launch_rmsnorm(ctx->proj, H, L.post_attn, c.epsilon, H, n, ctx->hidden, H, 1, ctx->stream, true));
    } else if (tp1) {
      if ((rc = gemv(ctx, L.o, ctx->att, ctx->q_l, nullptr, ctx->hidden, H, L.o_bias, EPI_ADD, n))) return rc;
    } else {
      if ((rc = gemv(ctx, L.o, ctx->att, ctx->q_l, nullptr, ctx->proj, H, L.o_bias, EPI_STORE, n))) return rc;
      if ((rc = tp_reduce_add(ctx, ctx->proj, ctx->hidden, n))) return rc;
    }
    const bool gated = gemma || c.ffn_gate;
    const int epi = !gated ? EPI_SILU : (c.activation == 1 || gemma) ? EPI_GLU_GELU : EPI_GLU_SILU;
    if ((rc = gemv(ctx, L.gate_up, ctx->hidden, H, L.ffn_norm, ctx->act, ctx->ffn_l, nullptr, epi, n))) return rc;
    if (gemma) {
      if ((rc = gemv(ctx, L.down, ctx->act, ctx->ffn_l, nullptr, ctx->proj, H, nullptr, EPI_STORE, n))) return rc;
      if (!tp1 && (rc = tp_allreduce_inplace(ctx->tp, ctx->proj, (size_t)n * H, ctx->stream, ctx->tp_spin_limit, &g_err))) return rc;
      CK(launch_rmsnorm(ctx->proj, H, L.post_ffw, c.epsilon, H, n, ctx->hidden, H, 1, ctx->stream, true));
    } else if (tp1) {
      if ((rc = gemv(ctx, L.down, ctx->act, ctx->ffn_l, nullptr, ctx->hidden, H, nullptr, EPI_ADD, n))) return rc;
    } else {
      if ((rc = gemv(ctx, L.down, ctx->act, ctx->ffn_l, nullptr, ctx->proj, H, nullptr, EPI_STORE, n))) return rc;
      if ((rc = tp_reduce_add(ctx, ctx->proj, ctx->hidden, n))) return rc;
    }
  }
  // LM head on the last row (engine.ts:177-178), then greedy argmax (engine.ts:305-309).
  float *logits_l = ctx->logits + ctx->vocab0;
  if ((rc = gemv(ctx, ctx->lm, ctx->hidden + (int64_t)(n - 1) * H, H, ctx->out_norm, logits_l, ctx->vocab_l, nullptr, EPI_STORE, 1)))
    return rc;
  CK(launch_argmax(logits_l, ctx->vocab_l, ctx->d_argmax, ctx->d_maxval, ctx->am_part, ctx->am_ctr, ctx->stream, true));
  if (!tp1) {
    if ((rc = tp_argmax_gather(ctx->tp, ctx->d_argmax, ctx->d_maxval, ctx->vocab0, ctx->stream, ctx->tp_spin_limit, &g_err))) return rc;
    if (want_logits_rows &&
        (rc = tp_gather_rows(ctx->tp, ctx->logits, ctx->c.vocab, ctx->vocab0, ctx->vocab_l, ctx->stream, ctx->tp_spin_limit, &g_err)))
      return rc;
  }
  if (io) CK(cudaMemcpyAsync(ctx->h_io + 1, ctx->d_argmax, sizeof(int32_t), cudaMemcpyDeviceToHost, ctx->stream));
  return WGD_OK;
}

// Draw of sample.cu over ctx->logits (whole vocabulary) into d_argmax, with the
// settings in d_sparams and the uniform d_uniform[step ? *step : 0].
static int enqueue_sample(wgd_ctx *ctx, const int *step) {
  SampleArgs s{};
  s.logits = ctx->logits;
  s.n = ctx->c.vocab;
  s.params = ctx->d_sparams;
  s.uniform = ctx->d_uniform;
  s.step = step;
  s.out = ctx->d_argmax;
  s.part = ctx->smp_part;
  s.ctr = ctx->smp_ctr;
  CK(launch_sample(s, ctx->sm_count, ctx->stream, true));
  ctx->kernels += 1;
  return WGD_OK;
}

// GenerationOptions rules of PagedEngine.generate (engine.ts:263-264).
static bool sampling_ok(double temperature, int top_k, double top_p) {
  return std::isfinite(temperature) && temperature >= 0 && temperature <= 2 && top_k >= 1 && top_k <= SAMPLE_MAX_K &&
         std::isfinite(top_p) && top_p > 0 && top_p <= 1;
}

static int forward_impl(wgd_ctx *ctx, const int32_t *ids, int n, int start, int want, int32_t *argmax_out, float *logits_out,
                        bool sampled);

extern "C" int wgd_forward(wgd_ctx *ctx, const int32_t *ids, int n, int start, int want, int32_t *argmax_out, float *logits_out) {
  return forward_impl(ctx, ids, n, start, want, argmax_out, logits_out, false);
}

extern "C" int wgd_forward_sample(wgd_ctx *ctx, const int32_t *ids, int n, int start, double temperature, int top_k, double top_p,
                                  double uniform, int32_t *token_out) {
  if (!ctx || !ids || !token_out) return fail(WGD_EINVAL, "null argument");
  if (!sampling_ok(temperature, top_k, top_p)) return fail(WGD_EINVAL, "Invalid sampling settings.");
  if (!(uniform >= 0 && uniform < 1)) return fail(WGD_EINVAL, "the uniform draw must lie in [0, 1)");
  if (temperature == 0) return forward_impl(ctx, ids, n, start, 1, token_out, nullptr, false);
  if (!ctx->ended) return fail(WGD_ESTATE, "Load a model first.");
  CK(cudaSetDevice(ctx->device));
  const SampleParams sp{temperature, top_p, top_k, 0};
  CK(cudaMemcpyAsync(ctx->d_sparams, &sp, sizeof(sp), cudaMemcpyHostToDevice, ctx->stream));
  CK(cudaMemcpyAsync(ctx->d_uniform, &uniform, sizeof(double), cudaMemcpyHostToDevice, ctx->stream));
  return forward_impl(ctx, ids, n, start, 1, token_out, nullptr, true);
}

static int forward_impl(wgd_ctx *ctx, const int32_t *ids, int n, int start, int want, int32_t *argmax_out, float *logits_out,
                        bool sampled) {
  if (!ctx || !ids) return fail(WGD_EINVAL, "null argument");
  if (!ctx->ended) return fail(WGD_ESTATE, "Load a model first.");
  std::string missing;
  if (!all_uploaded(ctx, &missing)) return fail(WGD_ESTATE, "weights not uploaded: " + missing);
  if (n < 1 || n > ctx->max_batch) return fail(WGD_EINVAL, "forward batch must be 1..max_batch");
  if (start < 0 || start + n > ctx->context) return fail(WGD_EINVAL, "positions exceed the context length");
  if (want < 0 || want > 2) return fail(WGD_EINVAL, "want must be 0, 1 or 2");
  for (int i = 0; i < n; i++)
    if (ids[i] < 0 || ids[i] >= ctx->c.vocab) return fail(WGD_EINVAL, "token id out of range");
  if (ctx->cancel.exchange(0)) return fail(WGD_ECANCELLED, "Stopped by user");
  CK(cudaSetDevice(ctx->device));
  ctx->st.streamed_bytes = 0;
  ctx->h_io[0] = start;
  memcpy(ctx->h_io + 2, ids, sizeof(int32_t) * n);
  CK(cudaEventRecord(ctx->ev0, ctx->stream));
  int rc;
  const bool gather_logits = want == 2 || (sampled && ctx->tp_size > 1);  // the draw reads the whole row on every rank
  const bool persist = n == 1 && ctx->persist_ok && ctx->persist_on && !(ctx->tp_size > 1 && (gather_logits || sampled));
  if (persist) {
    ctx->h_io[IO_CANCEL] = 0;
    if ((rc = enqueue_persist(ctx, ids[0], start, 1))) return rc;
    CK(cudaMemcpyAsync(ctx->h_io + 1, ctx->d_tokens, sizeof(int32_t), cudaMemcpyDeviceToHost, ctx->stream));
  } else if (n == 1 && ctx->graphs && !gather_logits && !ctx->paging) {
    if (!ctx->decode_exec) {
      CK(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
      rc = enqueue_forward(ctx, 1, false);
      cudaGraph_t g = nullptr;
      cudaError_t e = cudaStreamEndCapture(ctx->stream, &g);
      if (rc) { if (g) cudaGraphDestroy(g); return rc; }
      if (e != cudaSuccess) return fail(WGD_ECUDA, std::string("graph capture: ") + cudaGetErrorString(e));
      ctx->decode_graph = g;
      CK(cudaGraphInstantiate(&ctx->decode_exec, g, 0));
      ctx->decode_kernels = ctx->kernels;
    }
    CK(cudaGraphLaunch(ctx->decode_exec, ctx->stream));
    ctx->kernels = ctx->decode_kernels;
    ctx->st.kernel_launches += ctx->kernels;
  } else {
    if ((rc = enqueue_forward(ctx, n, gather_logits))) return rc;
    ctx->st.kernel_launches += ctx->kernels;
  }
  if (sampled) {
    const int before = ctx->kernels;
    if ((rc = enqueue_sample(ctx, nullptr))) return rc;
    ctx->st.kernel_launches += ctx->kernels - before;
    CK(cudaMemcpyAsync(ctx->h_io + 1, ctx->d_argmax, sizeof(int32_t), cudaMemcpyDeviceToHost, ctx->stream));
  }
  CK(cudaEventRecord(ctx->ev1, ctx->stream));
  if (want == 2 && logits_out) {
    if (ctx->tp_rank == 0) CK(cudaMemcpyAsync(logits_out, ctx->logits, sizeof(float) * ctx->c.vocab, cudaMemcpyDeviceToHost, ctx->stream));
  }
  CK(cudaStreamSynchronize(ctx->stream));
  float ms = 0.f;
  cudaEventElapsedTime(&ms, ctx->ev0, ctx->ev1);
  ctx->st.last_forward_ms = ms;
  ctx->st.forwards++;
  ctx->st.tokens += n;
  if (ctx->tp && tp_failed(ctx->tp)) return fail(WGD_ETIMEOUT, "a tensor-parallel peer did not answer within the wait limit");
  if (persist && (rc = persist_status(ctx))) return rc;
  if (ctx->h_io[IO_TC]) {
    ctx->h_io[IO_TC] = 0;
    return fail(WGD_ETIMEOUT, "a tensor-core GEMM pipeline wait ran out");
  }
  if (want >= 1) {
    if (ctx->h_io[1] < 0) return fail(WGD_ENONFINITE, "Inference produced non-finite logits. Stop and report this model/runtime combination.");
    if (argmax_out) *argmax_out = ctx->h_io[1];
  }
  return WGD_OK;
}

extern "C" int wgd_decode(wgd_ctx *ctx, int32_t first, int start, int steps, int32_t *tokens_out) {
  if (!ctx || !tokens_out) return fail(WGD_EINVAL, "null argument");
  if (!ctx->ended) return fail(WGD_ESTATE, "Load a model first.");
  std::string missing;
  if (!all_uploaded(ctx, &missing)) return fail(WGD_ESTATE, "weights not uploaded: " + missing);
  if (steps < 1 || start < 0 || start + steps > ctx->context) return fail(WGD_EINVAL, "positions exceed the context length");
  if (first < 0 || first >= ctx->c.vocab) return fail(WGD_EINVAL, "token id out of range");
  if (ctx->cancel.exchange(0)) return fail(WGD_ECANCELLED, "Stopped by user");
  CK(cudaSetDevice(ctx->device));
  int rc;
  if (ctx->persist_ok && ctx->persist_on) {
    ctx->h_io[IO_CANCEL] = 0;
    CK(cudaEventRecord(ctx->ev0, ctx->stream));
    if ((rc = enqueue_persist(ctx, first, start, steps))) return rc;
    CK(cudaEventRecord(ctx->ev1, ctx->stream));
    CK(cudaMemcpyAsync(tokens_out, ctx->d_tokens, sizeof(int32_t) * steps, cudaMemcpyDeviceToHost, ctx->stream));
    CK(cudaStreamSynchronize(ctx->stream));
    float ms = 0.f;
    cudaEventElapsedTime(&ms, ctx->ev0, ctx->ev1);
    const int done = ctx->h_io[IO_STATUS + 1];
    ctx->st.last_forward_ms = ms;
    ctx->st.forwards += done;
    ctx->st.tokens += done;
    return persist_status(ctx);
  }
  ctx->st.streamed_bytes = 0;
  if (!ctx->chain_exec && !ctx->paging) {
    CK(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
    rc = enqueue_forward(ctx, 1, false, false);
    if (!rc) {
      cudaError_t e = launch_advance(ctx->d_ids, ctx->d_start, ctx->d_argmax, ctx->d_tokens, ctx->d_step, ctx->d_err, ctx->stream, true);
      if (e != cudaSuccess) rc = fail(WGD_ECUDA, std::string("advance: ") + cudaGetErrorString(e));
      ctx->kernels += 1;
    }
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(ctx->stream, &g);
    if (rc) { if (g) cudaGraphDestroy(g); return rc; }
    if (e != cudaSuccess) return fail(WGD_ECUDA, std::string("graph capture: ") + cudaGetErrorString(e));
    ctx->chain_graph = g;
    CK(cudaGraphInstantiate(&ctx->chain_exec, g, 0));
    ctx->chain_kernels = ctx->kernels;
  }
  if (!ctx->paging) {
    ctx->kernels = ctx->chain_kernels;
    ctx->st.kernel_launches += (uint64_t)ctx->kernels * steps;
  }
  ctx->h_io[0] = start;
  ctx->h_io[2] = first;
  ctx->h_io[3] = 0;
  CK(cudaMemcpyAsync(ctx->d_start, ctx->h_io, sizeof(int32_t), cudaMemcpyHostToDevice, ctx->stream));
  CK(cudaMemcpyAsync(ctx->d_ids, ctx->h_io + 2, sizeof(int32_t), cudaMemcpyHostToDevice, ctx->stream));
  CK(cudaMemcpyAsync(ctx->d_step, ctx->h_io + 3, sizeof(int32_t), cudaMemcpyHostToDevice, ctx->stream));
  CK(cudaMemsetAsync(ctx->d_err, 0, sizeof(int32_t), ctx->stream));
  CK(cudaEventRecord(ctx->ev0, ctx->stream));
  if (ctx->paging) {  // paged weights: the same step enqueued per token (copy-stream events do not go in a graph)
    for (int i = 0; i < steps; i++) {
      if ((rc = enqueue_forward(ctx, 1, false, false))) return rc;
      CK(launch_advance(ctx->d_ids, ctx->d_start, ctx->d_argmax, ctx->d_tokens, ctx->d_step, ctx->d_err, ctx->stream, true));
      ctx->st.kernel_launches += (uint64_t)ctx->kernels + 1;
    }
  } else {
    for (int i = 0; i < steps; i++) CK(cudaGraphLaunch(ctx->chain_exec, ctx->stream));
  }
  CK(cudaEventRecord(ctx->ev1, ctx->stream));
  CK(cudaMemcpyAsync(tokens_out, ctx->d_tokens, sizeof(int32_t) * steps, cudaMemcpyDeviceToHost, ctx->stream));
  int32_t err = 0;
  CK(cudaMemcpyAsync(&err, ctx->d_err, sizeof(int32_t), cudaMemcpyDeviceToHost, ctx->stream));
  CK(cudaStreamSynchronize(ctx->stream));
  float ms = 0.f;
  cudaEventElapsedTime(&ms, ctx->ev0, ctx->ev1);
  ctx->st.last_forward_ms = ms;
  ctx->st.forwards += steps;
  ctx->st.tokens += steps;
  if (ctx->tp && tp_failed(ctx->tp)) return fail(WGD_ETIMEOUT, "a tensor-parallel peer did not answer within the wait limit");
  if (err == 2) return fail(WGD_ENONFINITE, "Inference produced non-finite logits. Stop and report this model/runtime combination.");
  return WGD_OK;
}

// wgd_decode with the draw of sample.cu in place of the argmax. The persistent kernel (when
// eligible) runs one token per launch, reading its input token and position from device
// memory; the draw and the advance step follow it on the stream, so there is no host round
// trip between tokens. Otherwise the per-kernel step, the draw and the advance step are
// captured once into a graph (settings and draws are device data, so it serves any of them).
extern "C" int wgd_decode_sample(wgd_ctx *ctx, int32_t first, int start, int steps, double temperature, int top_k, double top_p,
                                 const double *uniforms, int32_t *tokens_out) {
  if (!ctx || !tokens_out || !uniforms) return fail(WGD_EINVAL, "null argument");
  if (!sampling_ok(temperature, top_k, top_p)) return fail(WGD_EINVAL, "Invalid sampling settings.");
  if (temperature == 0) return wgd_decode(ctx, first, start, steps, tokens_out);
  if (!ctx->ended) return fail(WGD_ESTATE, "Load a model first.");
  std::string missing;
  if (!all_uploaded(ctx, &missing)) return fail(WGD_ESTATE, "weights not uploaded: " + missing);
  if (steps < 1 || start < 0 || start + steps > ctx->context) return fail(WGD_EINVAL, "positions exceed the context length");
  if (first < 0 || first >= ctx->c.vocab) return fail(WGD_EINVAL, "token id out of range");
  for (int i = 0; i < steps; i++)
    if (!(uniforms[i] >= 0 && uniforms[i] < 1)) return fail(WGD_EINVAL, "the uniform draws must lie in [0, 1)");
  if (ctx->cancel.exchange(0)) return fail(WGD_ECANCELLED, "Stopped by user");
  CK(cudaSetDevice(ctx->device));
  int rc;
  const SampleParams sp{temperature, top_p, top_k, 0};
  CK(cudaMemcpyAsync(ctx->d_sparams, &sp, sizeof(sp), cudaMemcpyHostToDevice, ctx->stream));
  CK(cudaMemcpyAsync(ctx->d_uniform, uniforms, sizeof(double) * steps, cudaMemcpyHostToDevice, ctx->stream));
  ctx->h_io[0] = start;
  ctx->h_io[2] = first;
  ctx->h_io[3] = 0;
  CK(cudaMemcpyAsync(ctx->d_start, ctx->h_io, sizeof(int32_t), cudaMemcpyHostToDevice, ctx->stream));
  CK(cudaMemcpyAsync(ctx->d_ids, ctx->h_io + 2, sizeof(int32_t), cudaMemcpyHostToDevice, ctx->stream));
  CK(cudaMemcpyAsync(ctx->d_step, ctx->h_io + 3, sizeof(int32_t), cudaMemcpyHostToDevice, ctx->stream));
  CK(cudaMemsetAsync(ctx->d_err, 0, sizeof(int32_t), ctx->stream));
  const bool persist = ctx->persist_ok && ctx->persist_on && ctx->tp_size == 1;  // the draw reads every rank's logits
  if (!persist && !ctx->chain_smp_exec && !ctx->paging) {
    CK(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
    rc = enqueue_forward(ctx, 1, ctx->tp_size > 1, false);
    if (!rc) rc = enqueue_sample(ctx, ctx->d_step);
    if (!rc) {
      cudaError_t e = launch_advance(ctx->d_ids, ctx->d_start, ctx->d_argmax, ctx->d_tokens, ctx->d_step, ctx->d_err, ctx->stream, true);
      if (e != cudaSuccess) rc = fail(WGD_ECUDA, std::string("advance: ") + cudaGetErrorString(e));
      ctx->kernels += 1;
    }
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(ctx->stream, &g);
    if (rc) { if (g) cudaGraphDestroy(g); return rc; }
    if (e != cudaSuccess) return fail(WGD_ECUDA, std::string("graph capture: ") + cudaGetErrorString(e));
    ctx->chain_smp_graph = g;
    CK(cudaGraphInstantiate(&ctx->chain_smp_exec, g, 0));
    ctx->chain_smp_kernels = ctx->kernels;
  }
  PersistArgs pa = ctx->pargs;
  if (persist) {
    ctx->h_io[IO_CANCEL] = 0;
    pa.dev_first = ctx->d_ids;
    pa.dev_start = ctx->d_start;
    pa.steps = 1;
    pa.tokens = ctx->d_ptok;
    CK(cudaMemsetAsync(pa.status, 0, 4 * sizeof(int), ctx->stream));
  }
  ctx->st.streamed_bytes = 0;
  CK(cudaEventRecord(ctx->ev0, ctx->stream));
  for (int i = 0; i < steps; i++) {
    if (persist) {
      if ((rc = persist_prepare(ctx, pa))) return rc;
      CK(launch_persist(pa, ctx->sm_count, ctx->stream));
      ctx->kernels = 1;
      if ((rc = enqueue_sample(ctx, ctx->d_step))) return rc;
      CK(launch_advance(ctx->d_ids, ctx->d_start, ctx->d_argmax, ctx->d_tokens, ctx->d_step, ctx->d_err, ctx->stream, true));
      ctx->kernels += 1;
      ctx->st.kernel_launches += ctx->kernels;
    } else if (ctx->paging) {
      if ((rc = enqueue_forward(ctx, 1, ctx->tp_size > 1, false))) return rc;
      if ((rc = enqueue_sample(ctx, ctx->d_step))) return rc;
      CK(launch_advance(ctx->d_ids, ctx->d_start, ctx->d_argmax, ctx->d_tokens, ctx->d_step, ctx->d_err, ctx->stream, true));
      ctx->kernels += 1;
      ctx->st.kernel_launches += ctx->kernels;
    } else {
      CK(cudaGraphLaunch(ctx->chain_smp_exec, ctx->stream));
      ctx->kernels = ctx->chain_smp_kernels;
      ctx->st.kernel_launches += ctx->kernels;
    }
  }
  CK(cudaEventRecord(ctx->ev1, ctx->stream));
  if (persist) CK(cudaMemcpyAsync(ctx->h_io + IO_STATUS, pa.status, 4 * sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
  CK(cudaMemcpyAsync(tokens_out, ctx->d_tokens, sizeof(int32_t) * steps, cudaMemcpyDeviceToHost, ctx->stream));
  int32_t err = 0;
  CK(cudaMemcpyAsync(&err, ctx->d_err, sizeof(int32_t), cudaMemcpyDeviceToHost, ctx->stream));
  CK(cudaStreamSynchronize(ctx->stream));
  float ms = 0.f;
  cudaEventElapsedTime(&ms, ctx->ev0, ctx->ev1);
  ctx->st.last_forward_ms = ms;
  ctx->st.forwards += steps;
  ctx->st.tokens += steps;
  if (ctx->tp && tp_failed(ctx->tp)) return fail(WGD_ETIMEOUT, "a tensor-parallel peer did not answer within the wait limit");
  if (persist && (rc = persist_status(ctx))) return rc;
  if (err == 2) return fail(WGD_ENONFINITE, "Inference produced non-finite logits. Stop and report this model/runtime combination.");
  return WGD_OK;
}

extern "C" int wgd_kernels_per_token(wgd_ctx *ctx, int *count) {
  if (!ctx || !count) return fail(WGD_EINVAL, "null argument");
  if (!ctx->ended) return fail(WGD_ESTATE, "Load a model first.");
  *count = ctx->kernels;
  return WGD_OK;
}

extern "C" int wgd_truncate_kv(wgd_ctx *ctx, int n_tokens) {
  if (!ctx) return fail(WGD_EINVAL, "null context");
  if (n_tokens < 0 || n_tokens > ctx->context) return fail(WGD_EINVAL, "token count outside the context");
  return WGD_OK;  // positions are explicit in every forward; later positions are overwritten
}

extern "C" void wgd_cancel(wgd_ctx *ctx) {
  if (!ctx) return;
  ctx->cancel.store(1);
  if (ctx->h_io) reinterpret_cast<volatile int32_t *>(ctx->h_io)[IO_CANCEL] = 1;  // polled by a running decode kernel
}

extern "C" int wgd_stats_get(wgd_ctx *ctx, wgd_stats *out) {
  if (!ctx || !out) return fail(WGD_EINVAL, "null argument");
  ctx->st.gpu_bytes = ctx->allocated;
  ctx->st.peak_gpu_bytes = ctx->peak;
  *out = ctx->st;
  return WGD_OK;
}

extern "C" int wgd_set_graphs(wgd_ctx *ctx, int enabled) {
  if (!ctx) return fail(WGD_EINVAL, "null context");
  ctx->graphs = enabled != 0;
  return WGD_OK;
}

extern "C" int wgd_set_prefill_gemm(wgd_ctx *ctx, int min_batch) {
  if (!ctx) return fail(WGD_EINVAL, "null context");
  if (min_batch < 0) return fail(WGD_EINVAL, "min_batch must be >= 0");
  ctx->tc_min_batch = min_batch;
  return WGD_OK;
}

extern "C" int wgd_set_persistent(wgd_ctx *ctx, int enabled) {
  if (!ctx) return fail(WGD_EINVAL, "null context");
  ctx->persist_on = enabled != 0;
  return WGD_OK;
}

extern "C" int wgd_persistent_status(wgd_ctx *ctx, char *why, int why_len) {
  if (!ctx) return fail(WGD_EINVAL, "null context");
  if (why && why_len > 0) snprintf(why, (size_t)why_len, "%s", ctx->persist_why.c_str());
  return ctx->persist_ok ? 1 : 0;
}

// ------------------------------------------------------------ tensor parallel

extern "C" int wgd_tp_handle_size(void) { return tp_handle_size(); }
extern "C" int wgd_tp_export(wgd_ctx *ctx, void *out) {
  if (!ctx || !out) return fail(WGD_EINVAL, "null argument");
  if (!ctx->tp) return fail(WGD_ESTATE, "tensor parallelism needs tp_size > 1 and model_end first");
  CK(cudaSetDevice(ctx->device));
  return tp_export(ctx->tp, out, &g_err);
}
extern "C" int wgd_tp_open_peers(wgd_ctx *ctx, const void *handles) {
  if (!ctx || !handles) return fail(WGD_EINVAL, "null argument");
  if (!ctx->tp) return fail(WGD_ESTATE, "tensor parallelism needs tp_size > 1 and model_end first");
  CK(cudaSetDevice(ctx->device));
  return tp_open(ctx->tp, handles, &g_err);
}
extern "C" int wgd_tp_set_timeout(wgd_ctx *ctx, uint64_t spin_limit) {
  if (!ctx) return fail(WGD_EINVAL, "null context");
  ctx->tp_spin_limit = spin_limit;
  return WGD_OK;
}

// ------------------------------------------------------------------ op entry points

namespace {
std::mutex g_op_mu;
unsigned *g_op_ctr[16] = {nullptr};
float *g_op_part[16] = {nullptr};
size_t g_op_part_n[16] = {0};
int g_op_sm[16] = {0};

int op_scratch(unsigned **ctr, int *sm) {
  int dev = 0;
  CK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 16) return fail(WGD_EINVAL, "device index");
  std::lock_guard<std::mutex> lk(g_op_mu);
  if (!g_op_ctr[dev]) {
    CK(cudaMalloc(&g_op_ctr[dev], sizeof(unsigned) * 4096));
    CK(cudaMemset(g_op_ctr[dev], 0, sizeof(unsigned) * 4096));
    cudaDeviceProp p;
    CK(cudaGetDeviceProperties(&p, dev));
    g_op_sm[dev] = p.multiProcessorCount;
  }
  *ctr = g_op_ctr[dev];
  *sm = g_op_sm[dev];
  return WGD_OK;
}
int op_part(size_t floats, float **out) {
  int dev = 0;
  CK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_op_mu);
  if (g_op_part_n[dev] < floats) {
    if (g_op_part[dev]) cudaFree(g_op_part[dev]);
    CK(cudaMalloc(&g_op_part[dev], floats * sizeof(float)));
    g_op_part_n[dev] = floats;
  }
  *out = g_op_part[dev];
  return WGD_OK;
}
}  // namespace

extern "C" int64_t wgd_dev_row_bytes(int type, int64_t cols) {
  if (!type_supported(type) || cols % block_elems(type)) return -1;
  return dev_row_bytes(type, cols);
}

extern "C" int wgd_op_repack(int type, int64_t rows, int64_t cols, const void *raw, void *packed, void *stream) {
  if (!type_supported(type) || cols % block_elems(type) || rows < 0) return fail(WGD_EINVAL, "bad type or shape");
  RowMap m{0, (int)rows, 0, 0, 0};
  CK(launch_repack(type, (const uint8_t *)raw, gguf_row_bytes(type, cols), 0, (int)rows, 0, (int)(cols / block_elems(type)),
                   (uint8_t *)packed, dev_row_bytes(type, cols), m, (cudaStream_t)stream));
  return WGD_OK;
}

extern "C" int wgd_op_dequant(int type, int64_t rows, int64_t cols, const void *packed, float *out, void *stream) {
  if (!type_supported(type) || cols % block_elems(type)) return fail(WGD_EINVAL, "bad type or shape");
  CK(launch_dequant(type, (const uint8_t *)packed, dev_row_bytes(type, cols), (int)rows, (int)cols, out, cols, (cudaStream_t)stream));
  return WGD_OK;
}

extern "C" int wgd_op_gemv(int type, int64_t rows, int64_t cols, const void *packed, const float *x, int batch, float *y,
                           void *stream) {
  if (!type_supported(type) || cols % block_elems(type) || cols % 32 || rows < 1 || batch < 1)
    return fail(WGD_EINVAL, "bad type, shape or batch");
  if (gemv_max_batch((int)cols) == 0) return fail(WGD_EINVAL, "matrix too wide for the GEMV kernel");
  unsigned *unused;
  int sm, rc;
  if ((rc = op_scratch(&unused, &sm))) return rc;  // caches the SM count of this device
  GemvArgs a{};
  a.w = (const uint8_t *)packed;
  a.drow = dev_row_bytes(type, cols);
  a.rows = (int)rows;
  a.cols = (int)cols;
  a.nb = (int)(cols / block_elems(type));
  a.x = x;
  a.ldx = (int)cols;
  a.y = y;
  a.ldy = (int)rows;
  a.epi = EPI_STORE;
  a.batch = batch;
  CK(launch_gemv(type, a, (cudaStream_t)stream, false, sm));
  return WGD_OK;
}

extern "C" int wgd_op_rmsnorm(const float *x, const float *w, int cols, int n, float eps, float *y, void *stream) {
  CK(launch_rmsnorm(x, cols, w, eps, cols, n, y, cols, 0, (cudaStream_t)stream, false));
  return WGD_OK;
}

extern "C" int wgd_op_rope(float *x, const float *norm_w, int n, int heads, int hd, int start, float theta, float scale, float eps,
                           int rotary_dim, int mode, void *stream) {
  if (hd % 2 || rotary_dim % 2 || rotary_dim > hd || heads < 1 || n < 1) return fail(WGD_EINVAL, "bad rope shape");
  RopeArgs a{};
  a.qkv = x;
  a.ld = heads * hd;
  a.n = n;
  a.heads = heads;
  a.kv_heads = 0;
  a.hd = hd;
  a.rot = rotary_dim ? rotary_dim : hd;
  a.mode = norm_w ? 0 : mode;
  a.q_norm = norm_w;
  a.eps = eps;
  a.theta = theta;
  a.scale = scale;
  a.start_host = start;
  a.capacity = 1;
  a.q_out = x;
  CK(launch_rope_kv(a, (cudaStream_t)stream, false));
  return WGD_OK;
}

extern "C" int wgd_op_attention(const float *q, const float *k, const float *v, float *out, int n, int heads, int kv_heads, int hd,
                                int start, float scale, int window, int capacity, void *stream) {
  if (n < 1 || heads < 1 || kv_heads < 1 || heads % kv_heads || heads / kv_heads > 8 || hd % 4 || hd > 512 || capacity < 1 ||
      window < 1 || start < 0)
    return fail(WGD_EINVAL, "bad attention shape");
  unsigned *ctr;
  int sm, rc;
  if ((rc = op_scratch(&ctr, &sm))) return rc;
  AttnArgs a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.out = out;
  a.n = n;
  a.heads = heads;
  a.kv_heads = kv_heads;
  a.hd = hd;
  a.capacity = capacity;
  a.window = window;
  a.scale = scale;
  a.start_host = start;
  a.splits = attention_splits(std::min(window, start + n));
  if (n * kv_heads > 2048) return fail(WGD_EINVAL, "too many attention rows for the op scratch");
  float *part;
  if ((rc = op_part(attention_part_floats(n, heads, kv_heads, hd, a.splits), &part))) return rc;
  a.part = part;
  a.ctr = ctr + 2048;
  CK(launch_attention(a, (cudaStream_t)stream, false));
  return WGD_OK;
}

extern "C" int wgd_op_argmax(const float *x, int n, int32_t *idx, void *stream) {
  if (n < 1) return fail(WGD_EINVAL, "empty input");
  unsigned *ctr;
  int sm, rc;
  if ((rc = op_scratch(&ctr, &sm))) return rc;
  float *part;
  if ((rc = op_part(2 * 256 + 4, &part))) return rc;
  CK(launch_argmax(x, n, idx, nullptr, part, ctr + 4000, (cudaStream_t)stream, false));
  return WGD_OK;
}

// ------------------------------------------------------------ tiled-layout ops

namespace {
float *g_t_part[16] = {nullptr};
size_t g_t_part_n[16] = {0};
unsigned *g_t_ctr[16] = {nullptr};
int g_t_ctr_n[16] = {0};
}  // namespace

extern "C" int64_t wgd_tiled_bytes(int type, int64_t rows, int64_t cols) {
  if (!tiled_type(type) || cols % 256 || rows < 1) return -1;
  return tiled_bytes(type, rows, cols);
}

extern "C" int wgd_op_repack_tiled(int type, int64_t rows, int64_t cols, const void *raw, void *tiled, void *stream) {
  if (!tiled_type(type) || cols % 256 || rows < 1) return fail(WGD_EINVAL, "tiled layout needs Q4_K/Q6_K and whole super-blocks");
  RowMap m{0, (int)rows, 0, 0, TILE_ROWS / 2};
  CK(launch_repack_tiled(type, (const uint8_t *)raw, gguf_row_bytes(type, cols), 0, (int)rows, 0, (int)(cols / 256),
                         (uint8_t *)tiled, (int)rows, m, (cudaStream_t)stream));
  return WGD_OK;
}

extern "C" int wgd_op_dequant_tiled(int type, int64_t rows, int64_t cols, const void *tiled, float *out, void *stream) {
  if (!tiled_type(type) || cols % 256) return fail(WGD_EINVAL, "tiled layout needs Q4_K/Q6_K and whole super-blocks");
  CK(launch_dequant_tiled(type, (const uint8_t *)tiled, (int)rows, (int)cols, out, cols, (cudaStream_t)stream));
  return WGD_OK;
}

extern "C" int wgd_op_gemv_tiled(int type, int64_t rows, int64_t cols, const void *tiled, const float *x, int batch, float *y,
                                 void *stream) {
  if (!tiled_type(type) || cols % 256 || rows < 1 || batch < 1 || gemv2_max_batch((int)cols) == 0)
    return fail(WGD_EINVAL, "bad type, shape or batch for the tiled GEMV");
  int dev = 0, sm = 0;
  unsigned *unused;
  int rc;
  if ((rc = op_scratch(&unused, &sm))) return rc;  // caches the SM count of this device
  CK(cudaGetDevice(&dev));
  const size_t need = gemv2_part_floats(type, (int)rows, (int)cols, sm);
  const int tiles = (int)((rows + 15) / 16);
  {
    std::lock_guard<std::mutex> lk(g_op_mu);
    if (g_t_part_n[dev] < need) {
      if (g_t_part[dev]) cudaFree(g_t_part[dev]);
      CK(cudaMalloc(&g_t_part[dev], need * sizeof(float)));
      g_t_part_n[dev] = need;
    }
    if (g_t_ctr_n[dev] < tiles) {
      if (g_t_ctr[dev]) cudaFree(g_t_ctr[dev]);
      CK(cudaMalloc(&g_t_ctr[dev], tiles * sizeof(unsigned)));
      CK(cudaMemset(g_t_ctr[dev], 0, tiles * sizeof(unsigned)));
      g_t_ctr_n[dev] = tiles;
    }
  }
  Gemv2Launch g{};
  g.w = (const uint8_t *)tiled;
  g.rows = (int)rows;
  g.cols = (int)cols;
  g.x = x;
  g.ldx = (int)cols;
  g.eps = 0.f;
  g.y = y;
  g.ldy = (int)rows;
  g.epi = EPI_STORE;
  g.batch = batch;
  g.part = g_t_part[dev];
  g.part_floats = g_t_part_n[dev];
  g.tile_ctr = g_t_ctr[dev];
  g.ctr_count = g_t_ctr_n[dev];
  CK(launch_gemv2(type, g, (cudaStream_t)stream, false, sm));
  return WGD_OK;
}
