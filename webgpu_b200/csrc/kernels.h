// Host-side launchers of the wgd CUDA kernels (internal; the public C ABI is include/wgd.h).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace wgd {

// ------------------------------------------------------------------ GEMV
// y[b, row] (op) acc(b, row) for the output rows of a weight matrix stored in the
// device row layout. Rows are processed in items of 4; `ctr` points to two
// zeroed uint32 (work ticket, finished CTAs) private to this launch site; the
// kernel leaves them zeroed again.
enum Epi : int {
  EPI_STORE = 0,     // y = acc + bias
  EPI_ADD = 1,       // y += acc + bias            (residual add)
  EPI_SILU = 2,      // y = silu(acc + bias)       (ungated MLP up projection)
  EPI_GLU_SILU = 3,  // rows interleaved [g g u u]: y = silu(g) * u
  EPI_GLU_GELU = 4,  // rows interleaved [g g u u]: y = gelu_tanh(g) * u
};
constexpr int GEMV_ROWS = 4;  // rows per work item; GLU interleave is 2 gate + 2 up rows

struct GemvArgs {
  const uint8_t *w;   // device-layout weights
  int64_t drow;       // bytes per device row
  int rows, cols;     // device rows (GLU: gate+up rows), columns
  int nb;             // blocks per row (for the scale arrays of Q4_0/Q8_0/Q6_K)
  const float *x;     // activations [batch][ldx]
  int ldx;
  const float *norm_w;  // non-null: x is RMS-normalised with this weight first
  float eps;
  float *y;
  int ldy;
  const float *bias;  // [rows] in device row order, or null
  int epi;
  int batch;          // number of activation rows
};
cudaError_t launch_gemv(int type, const GemvArgs &a, cudaStream_t s, bool pdl, int sm_count);
// Largest batch chunk the register-resident GEMV handles for this width in one pass.
int gemv_max_batch(int cols);

// ------------------------------------------------------- tensor-core GEMV
// Same operation over the tile-16 layout (tile.cuh) for Q4_K / Q6_K weights.
// `part`/`tile_ctr` are stream-K scratch: part_floats >= gemv2_part_floats(...),
// tile_ctr holds >= tiles zeroed counters (left zeroed).
struct Gemv2Launch {
  const uint8_t *w;
  int rows, cols;
  const float *x;
  int ldx;
  const float *norm_w;
  float eps;
  float *y;
  int ldy;
  const float *bias;
  int epi;
  int batch;
  float *part;
  size_t part_floats;
  unsigned *tile_ctr;
  int ctr_count;
};
cudaError_t launch_gemv2(int type, const Gemv2Launch &a, cudaStream_t s, bool pdl, int sm_count);
// Upper bound of the partial-sum floats one launch may need.
size_t gemv2_part_floats(int type, int rows, int cols, int sm_count);
// Largest activation chunk per pass (0 if the width is unsupported).
int gemv2_max_batch(int cols);

// ------------------------------------------------ prompt-batch tensor-core GEMM
// The same operation for a batch of activation rows on tcgen05 tensor cores
// (Q4_K / Q6_K in the tile-16 layout; gemm_tc.cu). Scratch: `panel` holds the prepared
// activations (gemm_tc_panel_bytes), `part` the partial sums of M-tiles cut
// between CTAs (gemm_tc_part_floats), `ctr` gemm_tc_mtiles(rows) zeroed
// counters (left zeroed). *status is set to 1 if a pipeline wait ran out.
constexpr int GEMM_TC_MAX_BATCH = 128;
struct GemmTcLaunch {
  int type;  // Q4_K or Q6_K
  const uint8_t *w;
  int rows, cols;
  const float *x;
  int ldx;
  const float *norm_w;
  float eps;
  float *y;
  int ldy;
  const float *bias;
  int epi;
  int batch;
  uint8_t *panel;
  float *part;
  unsigned *ctr;
  int *status;
};
cudaError_t launch_gemm_tc(const GemmTcLaunch &a, cudaStream_t s, int sm_count);
bool gemm_tc_supported(int type, int rows, int cols, int batch);
size_t gemm_tc_panel_bytes(int batch, int cols);
size_t gemm_tc_part_floats(int batch, int sm_count);
int gemm_tc_mtiles(int rows);

// --------------------------------------------------------------- layout
// Raw GGUF rows -> device rows. Source rows [0, nrows) at `src` (row stride
// `src_row_bytes`); block columns [blk0, blk0 + nbl) of each row are moved to
// destination row dst_row(r) = map(r0 + r) (see RowMap).
struct RowMap {
  int src_begin;   // first source row kept (global row index)
  int src_end;     // one past the last kept row
  int dst_base;    // logical destination row of src_begin
  int interleave;  // 0: plain; 1: gate part; 2: up part (GLU interleave)
  int glu_block;   // GLU interleave block R: device rows [R gate][R up] repeat
};
cudaError_t launch_repack(int type, const uint8_t *src, int64_t src_row_bytes, int row0, int nrows, int blk0, int nbl,
                          uint8_t *dst, int64_t dst_row_bytes, RowMap map, cudaStream_t s);
cudaError_t launch_dequant(int type, const uint8_t *w, int64_t drow, int rows, int cols, float *out, int64_t ldo,
                           cudaStream_t s);
// Tiled layout: same meaning; destination rows are placed in tiles of 16.
cudaError_t launch_repack_tiled(int type, const uint8_t *src, int64_t src_row_bytes, int row0, int nrows, int blk0, int nbl,
                                uint8_t *dst, int dst_rows, RowMap map, cudaStream_t s);
cudaError_t launch_dequant_tiled(int type, const uint8_t *w, int rows, int cols, float *out, int64_t ldo, cudaStream_t s);
// Dequantises selected rows (ids[t]) scaled by `scale` into out[t][cols] (embedding gather).
cudaError_t launch_embed(int type, const uint8_t *w, int64_t drow, int cols, const int *ids, int n, int vocab, float scale,
                         float *out, int ldo, int *err, cudaStream_t s, bool pdl, bool tiled = false);

// ---------------------------------------------------------- block ops
// RMS norm of x rows (n rows of `cols`) with weight w: y = x * rsqrt(mean(x^2)+eps) * w.
// add != 0: y += (normed value) instead (Gemma post-norm residual).
cudaError_t launch_rmsnorm(const float *x, int ldx, const float *w, float eps, int cols, int n, float *y, int ldy, int add,
                           cudaStream_t s, bool pdl);

struct RopeArgs {
  float *qkv;          // [n][ld] rows: q heads, then k heads, then v heads (hd each)
  int ld;
  int n, heads, kv_heads, hd;
  int rot;             // rotary dims (even, <= hd)
  int mode;            // 0 half-split, 1 adjacent pairs
  const float *q_norm, *k_norm;  // per-head RMS weights (qk-norm) or null
  float eps;
  double theta, scale;
  const float2 *table; // (cos, sin) of pos*scale/theta^(2i/rot), [context][rot/2]; null: computed in double
  const int *start;    // device int: absolute position of row 0
  int start_host;      // used when start == nullptr
  float *k_cache, *v_cache;  // [kv_heads][capacity][hd]
  int capacity;
  float *q_out;        // [n][heads][hd]
};
cudaError_t launch_rope_kv(const RopeArgs &a, cudaStream_t s, bool pdl);

struct AttnArgs {
  const float *q;      // [n][heads][hd]
  const float *k, *v;  // [kv_heads][capacity][hd]
  float *out;          // [n][heads][hd]
  int n, heads, kv_heads, hd, capacity, window;
  float scale;
  const int *start;    // device int or null (then start_host)
  int start_host;
  float *part;         // scratch: [n][kv_heads][splits][group][hd + 4] (16-byte aligned)
  unsigned *ctr;       // [n * kv_heads] zeroed counters (left zeroed)
  int splits;          // grid.y
  // decode (n == 1) with the RoPE/KV write fused in: q/k/v are read raw from `qkv`,
  // rotated (after the optional per-head norm) with `table`, and the new K/V row is
  // written to ring slot start % capacity of k/v by the CTA that owns that position.
  const float *qkv;    // non-null: fused mode; row 0 = q heads | k heads | v heads
  const float *q_norm, *k_norm;
  float eps;
  int rot, mode;
  const float2 *table;
};
cudaError_t launch_attention(const AttnArgs &a, cudaStream_t s, bool pdl);
int attention_splits(int max_len);
size_t attention_part_floats(int n, int heads, int kv_heads, int hd, int splits);

// Argmax over finite values of x[0..n) (first index wins ties). Writes
// out_idx (int, -1 when nothing is finite) and out_val. `part` holds
// 2*blocks floats; ctr one zeroed uint32.
cudaError_t launch_argmax(const float *x, int n, int *out_idx, float *out_val, float *part, unsigned *ctr, cudaStream_t s,
                          bool pdl);
int argmax_blocks(int n);

// Temperature / top-k / top-p draw over one row of logits (sample.cu). Settings and
// the uniform draws live in device memory so that a captured graph serves any of them.
constexpr int SAMPLE_MAX_K = 200;     // the reference's largest topK
constexpr int SAMPLE_MAX_GRID = 256;  // CTAs of one launch (part holds GRID * top_k keys)
struct SampleParams {
  double temperature;  // > 0 draws, == 0 greedy
  double top_p;        // nucleus mass in (0, 1]
  int top_k;           // 1..SAMPLE_MAX_K
  int pad;
};
struct SampleArgs {
  const float *logits;
  int n;
  const SampleParams *params;
  const double *uniform;  // uniform[step ? *step : 0], in [0, 1)
  const int *step;
  int *out;               // token; -1 when no logit is finite
  uint64_t *part;         // SAMPLE_MAX_GRID * SAMPLE_MAX_K keys
  unsigned *ctr;          // one zeroed counter (left zeroed)
};
cudaError_t launch_sample(const SampleArgs &a, int sm_count, cudaStream_t s, bool pdl);
int sample_grid(int n, int sm_count);

// Device decode loop step: ids[0] = *argmax; *start += 1; tokens[*step] = *argmax; ++*step.
// A non-finite row (argmax -1) sets *err and feeds token 0.
cudaError_t launch_advance(int *ids, int *start, const int *argmax, int *tokens, int *step, int *err, cudaStream_t s, bool pdl);

// Elementwise: y += x (n floats).
cudaError_t launch_add(const float *x, float *y, int64_t n, cudaStream_t s, bool pdl);

}  // namespace wgd
