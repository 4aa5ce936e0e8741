/*
 * CPU oracle for the decoder hot path — TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the reference runtime's CPU arithmetic so that
 * the CUDA library can be checked against it. It is never linked into the
 * product library; only the tests, the smoke check and the CPU-baseline leg of
 * the benchmark load it (as oracle/_build/liboracle.so).
 *
 * What it follows (paths inside the reference project, ahpah-dev/WebGPU 0.9.0):
 *   - halfToFloat / decodeWeight          src/core/quant.ts:2-29   (f64, exactly as written)
 *   - fp32 dequant twin in WGSL order     src/core/shaders.ts:13-38 (weightFunction)
 *   - packed matmul expectation           src/verify.ts:32-35
 *   - greedy sample                       src/core/engine.ts:305-309
 *   - temperature / top-k / top-p sample  src/core/engine.ts:305-324 (the branch at 310-323)
 *   - RMSNorm / RoPE / attention fixtures src/verify.ts:39-66, src/verify-context.ts:8-41,
 *                                         src/core/shaders.ts:55-122,139-169
 *   - the float64 CPU decoder             scripts/verify-dense.mjs:138-211
 *     extended with the engine's block    src/core/engine.ts:138-180,217-251 (bias, output
 *     rules                               bias, ungated MLP, sliding window, rope scale, partial
 *                                         rotary) and the Gemma block engine.ts:158-174
 *                                         (post norms, GELU-tanh GLU shaders.ts:136,
 *                                         sqrt(hidden) embedding scale engine.ts:143,
 *                                         local/global theta and window engine.ts:147,161,163).
 *
 * Pinning: the dequant functions are checked against the known-answer tests of
 * tests/quant.test.ts:6-45 (restated in tests/test_oracle_quant.py). The decoder
 * is cross-checked against an independent float64 transformer implementation.
 *
 * Build: -O2 -ffp-contract=off (no FMA contraction anywhere), -fopenmp.
 */
#include <math.h>
#include <stdio.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14 };

/* ------------------------------------------------------------------ dequant */

/* quant.ts:2-5 */
double or_half_to_float(uint32_t h) {
  double sign = (h & 0x8000) ? -1.0 : 1.0;
  int exponent = (h >> 10) & 31, fraction = h & 1023;
  if (exponent == 0) return sign * ldexp(1.0, -14) * fraction / 1024.0;
  if (exponent == 31) return fraction ? NAN : sign * INFINITY;
  return sign * ldexp(1.0, exponent - 15) * (1.0 + fraction / 1024.0);
}

/* quant.ts:6-29 — the GGML block layouts, decoded element by element in f64. */
double or_decode_weight(const uint8_t *b, int type, int64_t i) {
#define F16(p) or_half_to_float((uint32_t)b[(p)] | ((uint32_t)b[(p) + 1] << 8))
  if (type == T_F32) { float f; memcpy(&f, b + i * 4, 4); return f; }
  if (type == T_F16) return F16(i * 2);
  if (type == T_Q4_0) {
    int64_t p = (i / 32) * 18; int j = (int)(i % 32);
    return F16(p) * (double)(((b[p + 2 + j % 16] >> (j < 16 ? 0 : 4)) & 15) - 8);
  }
  if (type == T_Q8_0) {
    int64_t p = (i / 32) * 34; int q = b[p + 2 + i % 32];
    return F16(p) * (double)(q > 127 ? q - 256 : q);
  }
  if (type == T_Q4_K || type == T_Q5_K) {
    int64_t p = (i / 256) * (type == T_Q4_K ? 144 : 176); int j = (int)(i % 256), s = j / 32;
    int sc = s < 4 ? (b[p + 4 + s] & 63) : ((b[p + 8 + s] & 15) | ((b[p + s] >> 6) << 4));
    int mn = s < 4 ? (b[p + 8 + s] & 63) : ((b[p + 8 + s] >> 4) | ((b[p + 4 + s] >> 6) << 4));
    int q = (b[p + (type == T_Q4_K ? 16 : 48) + (j / 64) * 32 + j % 32] >> (s % 2 * 4)) & 15;
    if (type == T_Q5_K) q |= ((b[p + 16 + j % 32] >> s) & 1) << 4;
    /* JS evaluates f16(p) * sc * q - f16(p + 2) * mn left to right in doubles. */
    return F16(p) * sc * q - F16(p + 2) * mn;
  }
  if (type == T_Q6_K) {
    int64_t p = (i / 256) * 210; int j = (int)(i % 256);
    int segment = j / 128, quarter = (j % 128) / 32, lane = j % 32;
    int low = (b[p + segment * 64 + quarter % 2 * 32 + lane] >> ((quarter / 2) * 4)) & 15;
    int high = (b[p + 128 + segment * 32 + lane] >> (quarter * 2)) & 3;
    int scale = b[p + 192 + segment * 8 + quarter * 2 + lane / 16];
    return F16(p + 208) * (double)(scale > 127 ? scale - 256 : scale) * (double)((low | high << 4) - 32);
  }
#undef F16
  return NAN;
}

/* shaders.ts:44-63 — the same values in the WGSL shader's f32 operation order,
 * with every product and difference rounded separately (no contraction). */
static float hf(const uint8_t *b, int64_t p) { return (float)or_half_to_float((uint32_t)b[p] | ((uint32_t)b[p + 1] << 8)); }
float or_decode_weight_f32(const uint8_t *b, int type, int64_t i) {
  if (type == T_F32) { float f; memcpy(&f, b + i * 4, 4); return f; }
  if (type == T_F16) return hf(b, i * 2);
  if (type == T_Q4_0) {
    int64_t p = (i / 32) * 18; int j = (int)(i % 32);
    return hf(b, p) * (float)((int)((b[p + 2 + j % 16] >> ((j / 16) * 4)) & 15) - 8);
  }
  if (type == T_Q8_0) {
    int64_t p = (i / 32) * 34; int q = (int8_t)b[p + 2 + i % 32];
    return hf(b, p) * (float)q;
  }
  if (type == T_Q4_K || type == T_Q5_K) {
    int64_t p = (i / 256) * (type == T_Q4_K ? 144 : 176); int j = (int)(i % 256), s = j / 32;
    unsigned sc, mn;
    if (s < 4) { sc = b[p + 4 + s] & 63u; mn = b[p + 8 + s] & 63u; }
    else { sc = (b[p + 8 + s] & 15u) | ((b[p + s] >> 6u) << 4u); mn = (b[p + 8 + s] >> 4u) | ((b[p + 4 + s] >> 6u) << 4u); }
    unsigned q = (b[p + (type == T_Q4_K ? 16 : 48) + (j / 64) * 32 + j % 32] >> ((s % 2) * 4)) & 15u;
    if (type == T_Q5_K) q |= ((b[p + 16 + j % 32] >> s) & 1u) << 4u;
    volatile float a = hf(b, p) * (float)(sc * q);
    volatile float c = hf(b, p + 2) * (float)mn;
    return a - c;
  }
  if (type == T_Q6_K) {
    int64_t p = (i / 256) * 210; int j = (int)(i % 256);
    int segment = j / 128, quarter = (j % 128) / 32, lane = j % 32;
    unsigned low = (b[p + segment * 64 + (quarter % 2) * 32 + lane] >> ((quarter / 2) * 4)) & 15u;
    unsigned high = (b[p + 128 + segment * 32 + lane] >> (quarter * 2)) & 3u;
    int8_t sc = (int8_t)b[p + 192 + segment * 8 + quarter * 2 + lane / 16];
    volatile float ds = hf(b, p + 208) * (float)sc;
    return ds * (float)((int)(low | (high << 4)) - 32);
  }
  return NAN;
}

int64_t or_block_elems(int type) {
  switch (type) { case T_F32: case T_F16: return 1; case T_Q4_0: case T_Q8_0: return 32; default: return 256; }
}
int64_t or_block_bytes(int type) {
  switch (type) {
    case T_F32: return 4; case T_F16: return 2; case T_Q4_0: return 18; case T_Q8_0: return 34;
    case T_Q4_K: return 144; case T_Q5_K: return 176; case T_Q6_K: return 210; default: return 0;
  }
}
int64_t or_row_bytes(int type, int64_t cols) { return cols / or_block_elems(type) * or_block_bytes(type); }

/* Element-wise loops over the restated functions (no shortcuts: each value is
 * produced by the quant.ts formula). */
void or_dequant(const uint8_t *data, int type, int64_t n, double *out) {
  for (int64_t i = 0; i < n; i++) out[i] = or_decode_weight(data, type, i);
}
void or_dequant_f32(const uint8_t *data, int type, int64_t n, float *out) {
  for (int64_t i = 0; i < n; i++) out[i] = or_decode_weight_f32(data, type, i);
}

/* Row dequant used by the decoder and the matmul: the quant.ts formula of
 * or_decode_weight per element, with the per-block operands (d, dmin, the
 * 6-bit scale and min, the int8 scale) hoisted out of the element loop. Every
 * value is the same expression on the same operands, so the result is
 * bit-identical to or_decode_weight (checked by or_dequant_row_matches). */
static void dequant_row(const uint8_t *b, int type, int64_t cols, double *out) {
#define F16(p) or_half_to_float((uint32_t)b[(p)] | ((uint32_t)b[(p) + 1] << 8))
  if (type == T_F32) { for (int64_t i = 0; i < cols; i++) { float f; memcpy(&f, b + i * 4, 4); out[i] = f; } return; }
  if (type == T_F16) { for (int64_t i = 0; i < cols; i++) out[i] = F16(i * 2); return; }
  if (type == T_Q4_0) {
    for (int64_t k = 0; k < cols / 32; k++) {
      int64_t p = k * 18; double d = F16(p);
      for (int j = 0; j < 32; j++) out[k * 32 + j] = d * (double)(((b[p + 2 + j % 16] >> (j < 16 ? 0 : 4)) & 15) - 8);
    }
    return;
  }
  if (type == T_Q8_0) {
    for (int64_t k = 0; k < cols / 32; k++) {
      int64_t p = k * 34; double d = F16(p);
      for (int j = 0; j < 32; j++) { int q = b[p + 2 + j]; out[k * 32 + j] = d * (double)(q > 127 ? q - 256 : q); }
    }
    return;
  }
  if (type == T_Q4_K || type == T_Q5_K) {
    const int bb = type == T_Q4_K ? 144 : 176, qo = type == T_Q4_K ? 16 : 48;
    for (int64_t k = 0; k < cols / 256; k++) {
      int64_t p = k * bb; double d = F16(p), dm = F16(p + 2);
      for (int s = 0; s < 8; s++) {
        int sc = s < 4 ? (b[p + 4 + s] & 63) : ((b[p + 8 + s] & 15) | ((b[p + s] >> 6) << 4));
        int mn = s < 4 ? (b[p + 8 + s] & 63) : ((b[p + 8 + s] >> 4) | ((b[p + 4 + s] >> 6) << 4));
        for (int jj = 0; jj < 32; jj++) {
          int j = 32 * s + jj;
          int q = (b[p + qo + (j / 64) * 32 + j % 32] >> (s % 2 * 4)) & 15;
          if (type == T_Q5_K) q |= ((b[p + 16 + j % 32] >> s) & 1) << 4;
          out[k * 256 + j] = d * sc * q - dm * mn;
        }
      }
    }
    return;
  }
  if (type == T_Q6_K) {
    for (int64_t k = 0; k < cols / 256; k++) {
      int64_t p = k * 210; double d = F16(p + 208);
      for (int j = 0; j < 256; j++) {
        int segment = j / 128, quarter = (j % 128) / 32, lane = j % 32;
        int low = (b[p + segment * 64 + quarter % 2 * 32 + lane] >> ((quarter / 2) * 4)) & 15;
        int high = (b[p + 128 + segment * 32 + lane] >> (quarter * 2)) & 3;
        int scale = b[p + 192 + segment * 8 + quarter * 2 + lane / 16];
        out[k * 256 + j] = d * (double)(scale > 127 ? scale - 256 : scale) * (double)((low | high << 4) - 32);
      }
    }
    return;
  }
#undef F16
  for (int64_t i = 0; i < cols; i++) out[i] = NAN;
}

/* 1 when the hoisted row decoder reproduces or_decode_weight bit for bit. */
int or_dequant_row_matches(const uint8_t *row, int type, int64_t cols) {
  double *a = (double *)malloc(sizeof(double) * cols);
  dequant_row(row, type, cols, a);
  int ok = 1;
  for (int64_t i = 0; i < cols && ok; i++) {
    double r = or_decode_weight(row, type, i);
    ok = memcmp(&a[i], &r, sizeof(double)) == 0;
  }
  free(a);
  return ok;
}

static int g_threads = 1;
void or_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
int or_get_threads(void) { return g_threads; }

/* verify.ts:32-35: y[b*stride + rowBase + r] = sum_c decode(W, r*cols + c) * x[(b+inOff)*cols + c],
 * accumulated in f64 in column order. */
void or_matmul(const uint8_t *w, int type, int64_t rows, int64_t cols, const float *x, int batch,
               int64_t stride, int64_t row_base, int input_offset, double *y) {
  int64_t rb = or_row_bytes(type, cols);
#pragma omp parallel num_threads(g_threads)
  {
    double *buf = (double *)malloc(sizeof(double) * cols);
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
      dequant_row(w + r * rb, type, cols, buf);
      for (int b = 0; b < batch; b++) {
        const float *xb = x + (int64_t)(b + input_offset) * cols;
        double sum = 0;
        for (int64_t c = 0; c < cols; c++) sum += buf[c] * (double)xb[c];
        y[(int64_t)b * stride + row_base + r] = sum;
      }
    }
    free(buf);
  }
}

/* engine.ts:305-309: first finite maximum; -1 when no value is finite. */
int64_t or_greedy(const float *logits, int64_t n) {
  double best = -INFINITY; int64_t id = -1;
  for (int64_t i = 0; i < n; i++) if (isfinite(logits[i]) && logits[i] > best) { best = logits[i]; id = i; }
  return id;
}
int64_t or_greedy_f64(const double *logits, int64_t n) {
  double best = -INFINITY; int64_t id = -1;
  for (int64_t i = 0; i < n; i++) if (isfinite(logits[i]) && logits[i] > best) { best = logits[i]; id = i; }
  return id;
}

/* engine.ts:305-324 (temperature > 0), step for step: a candidate list kept sorted by
 * value (a new value goes after the equal ones, as JS's stable sort leaves it), a
 * finite logit enters while the list is short or when it beats the last entry, the
 * entry past top_k is dropped; probability exp((v - best) / temperature) in double;
 * total and the nucleus mass summed in list order; draw = uniform * retained,
 * subtracted in list order. `uniform` stands for Math.random(). Returns -1 when no
 * logit is finite (the reference throws). temperature == 0 is or_greedy. */
int64_t or_sample(const float *logits, int64_t n, double temperature, int top_k, double top_p, double uniform) {
  const int64_t best_id = or_greedy(logits, n);
  if (best_id < 0) return -1;
  if (temperature == 0) return best_id;
  const double best = logits[best_id];
  int64_t *id = malloc(sizeof(int64_t) * (size_t)(top_k + 1));
  double *val = malloc(sizeof(double) * (size_t)(top_k + 1)), *prob = malloc(sizeof(double) * (size_t)(top_k + 1));
  int count = 0;
  for (int64_t i = 0; i < n; i++) {
    if (!isfinite(logits[i])) continue;
    const double v = logits[i];
    if (count < top_k || v > val[count - 1]) {
      int at = count;
      while (at > 0 && val[at - 1] < v) at--;
      for (int j = count; j > at; j--) { id[j] = id[j - 1]; val[j] = val[j - 1]; prob[j] = prob[j - 1]; }
      id[at] = i; val[at] = v; prob[at] = exp((v - best) / temperature);
      if (++count > top_k) count--;
    }
  }
  double total = 0;
  for (int j = 0; j < count; j++) total += prob[j];
  double retained = 0;
  int cutoff = 0;
  for (; cutoff < count; cutoff++) {
    retained += prob[cutoff];
    if (retained / total >= top_p) { cutoff++; break; }
  }
  double draw = uniform * retained;
  int64_t out = best_id;
  for (int j = 0; j < cutoff; j++) {
    draw -= prob[j];
    if (draw <= 0) { out = id[j]; break; }
  }
  free(id); free(val); free(prob);
  return out;
}

/* ------------------------------------------------------- primitive references */

/* shaders.ts:55-68 (normShader), in f64: y = x * rsqrt(mean(x^2) + eps) * w per row. */
void or_rmsnorm(const float *x, const float *w, int64_t n, int64_t rows, double eps, double *y) {
  for (int64_t r = 0; r < rows; r++) {
    double sum = 0;
    for (int64_t i = 0; i < n; i++) sum += (double)x[r * n + i] * x[r * n + i];
    double inv = 1.0 / sqrt(sum / n + eps);
    for (int64_t i = 0; i < n; i++) y[r * n + i] = x[r * n + i] * inv * w[i];
  }
}

/* Rotary embedding on one head vector (f64, in place).
 * mode 0: half-split pairs (i, i+rot/2) — ropeNeoxShader shaders.ts:139-154 / verify-dense rotate 'neox'
 * mode 1: adjacent pairs (2i, 2i+1)   — ropeClassicShader shaders.ts:155-169 / verify-dense rotate 'norm'
 * angle = pos * scale / theta^(2i/rot), verify-dense.mjs:149-159. */
static void rotate_head(double *x, int hd, int rot, int mode, double pos, double scale, double theta) {
  if (rot == 0) rot = hd;
  for (int j = 0; j < rot / 2; j++) {
    double angle = pos * scale / pow(theta, (2.0 * j) / rot);
    double c = cos(angle), s = sin(angle);
    int a = mode == 0 ? j : 2 * j, b = mode == 0 ? j + rot / 2 : 2 * j + 1;
    double left = x[a], right = x[b];
    x[a] = left * c - right * s;
    x[b] = left * s + right * c;
  }
}
/* verify-dense.mjs:160-164 rmsHead, f64 in place. */
static void rms_head(double *x, const double *w, int hd, double eps) {
  double sum = 0;
  for (int d = 0; d < hd; d++) sum += x[d] * x[d];
  double inv = 1.0 / sqrt(sum / hd + eps);
  for (int d = 0; d < hd; d++) x[d] = x[d] * inv * w[d];
}

/* Rope op reference over x[n][heads][hd] (f32 in, f64 out), position of row t = start + t.
 * qk_norm != 0 follows ropeShader (shaders.ts:69-87): per-head RMS norm with weight w,
 * then half-split rotation of the first rot dims; the tail keeps the normalised value. */
void or_rope(const float *x, const float *w, int n, int heads, int hd, int start, double theta, double scale,
             double eps, int rot, int mode, int qk_norm, double *y) {
  double *wd = (double *)malloc(sizeof(double) * hd);
  for (int d = 0; d < hd; d++) wd[d] = w ? w[d] : 1.0;
  for (int t = 0; t < n; t++)
    for (int h = 0; h < heads; h++) {
      double *v = y + ((int64_t)t * heads + h) * hd;
      for (int d = 0; d < hd; d++) v[d] = x[((int64_t)t * heads + h) * hd + d];
      if (qk_norm) rms_head(v, wd, hd, eps);
      rotate_head(v, hd, rot, qk_norm ? 0 : mode, (double)(start + t), scale, theta);
    }
  free(wd);
}

/* attentionShader semantics (shaders.ts:88-122; expectation as verify.ts:47-52 and
 * verify-context.ts:30-41): query row t at absolute position start+t attends keys
 * [end - min(end, window), end), end = start+t+1, read from ring slot (pos % capacity)
 * of a cache laid out [capacity][kv_heads][hd]. f64 softmax. */
void or_attention(const float *q, const float *k, const float *v, int n, int heads, int kv_heads, int hd,
                  int start, double scale, int window, int capacity, double *y) {
  int group = heads / kv_heads;
  for (int t = 0; t < n; t++)
    for (int h = 0; h < heads; h++) {
      int64_t end = start + t + 1, begin = end - (end < window ? end : window);
      int kh = h / group;
      const float *qv = q + ((int64_t)t * heads + h) * hd;
      double maximum = -INFINITY;
      double *scores = (double *)malloc(sizeof(double) * (end - begin));
      for (int64_t p = begin; p < end; p++) {
        const float *kv = k + ((p % capacity) * kv_heads + kh) * hd;
        double dot = 0;
        for (int d = 0; d < hd; d++) dot += (double)qv[d] * kv[d];
        scores[p - begin] = dot * scale;
        if (scores[p - begin] > maximum) maximum = scores[p - begin];
      }
      double total = 0;
      for (int64_t p = begin; p < end; p++) { scores[p - begin] = exp(scores[p - begin] - maximum); total += scores[p - begin]; }
      for (int d = 0; d < hd; d++) {
        double sum = 0;
        for (int64_t p = begin; p < end; p++) sum += scores[p - begin] / total * v[((p % capacity) * kv_heads + kh) * hd + d];
        y[((int64_t)t * heads + h) * hd + d] = sum;
      }
      free(scores);
    }
}

/* ---------------------------------------------------------------- decoder */

typedef struct or_config {
  int32_t family;          /* 0: dense llama/qwen2/qwen3/mistral, 1: gemma3 */
  int32_t hidden, intermediate, layers, heads, kv_heads, head_dim, vocab;
  double epsilon, theta, local_theta;
  int32_t window, period;  /* Gemma local window and layer period (gguf.ts:131,133) */
  double attention_scale, rope_scale;
  int32_t rotary_dim;
  int32_t rope_mode;       /* 0: neox (half split), 1: norm (adjacent pairs) */
  int32_t sliding_window;  /* dense families: 0 = full context */
  int32_t qk_norm, ffn_gate, activation; /* activation 0 silu, 1 gelu */
  int32_t bias_q, bias_k, bias_v, bias_output;
  int32_t context;
} or_config;

typedef struct { const uint8_t *data; int type; int64_t cols, rows; double *vec; } or_tensor;

enum { W_ATTN_NORM, W_Q, W_K, W_V, W_O, W_QB, W_KB, W_VB, W_OB, W_QN, W_KN, W_POST_ATTN, W_FFN_NORM,
       W_GATE, W_UP, W_DOWN, W_POST_FFW, W_COUNT };
static const char *LAYER_NAMES[W_COUNT] = {
  "attn_norm.weight", "attn_q.weight", "attn_k.weight", "attn_v.weight", "attn_output.weight",
  "attn_q.bias", "attn_k.bias", "attn_v.bias", "attn_output.bias", "attn_q_norm.weight", "attn_k_norm.weight",
  "post_attention_norm.weight", "ffn_norm.weight", "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight",
  "post_ffw_norm.weight"};

typedef struct or_model {
  or_config c;
  or_tensor embd, out_norm, output;
  or_tensor *layer; /* layers * W_COUNT */
} or_model;

typedef struct or_state { int context; double **k, **v; /* per layer [context][kv_heads*hd] */ } or_state;

or_model *or_model_create(const or_config *cfg) {
  or_model *m = (or_model *)calloc(1, sizeof(or_model));
  m->c = *cfg;
  m->layer = (or_tensor *)calloc((size_t)cfg->layers * W_COUNT, sizeof(or_tensor));
  return m;
}

static void free_tensor(or_tensor *t) { free(t->vec); t->vec = NULL; }
void or_model_destroy(or_model *m) {
  if (!m) return;
  free_tensor(&m->embd); free_tensor(&m->out_norm); free_tensor(&m->output);
  for (int i = 0; i < m->c.layers * W_COUNT; i++) free_tensor(&m->layer[i]);
  free(m->layer); free(m);
}

/* Registers a tensor by its GGUF name. `data` is borrowed (GGUF bytes) and must
 * outlive the model. 1-D tensors (norms, biases) are decoded once, as
 * engine.ts:102-109 does on load. Returns 0, or -1 for an unknown name. */
int or_model_set(or_model *m, const char *name, const uint8_t *data, int type, int64_t cols, int64_t rows) {
  or_tensor t = {data, type, cols, rows, NULL};
  if (rows == 1) { t.vec = (double *)malloc(sizeof(double) * cols); or_dequant(data, type, cols, t.vec); }
  if (!strcmp(name, "token_embd.weight")) { m->embd = t; return 0; }
  if (!strcmp(name, "output_norm.weight")) { m->out_norm = t; return 0; }
  if (!strcmp(name, "output.weight")) { m->output = t; return 0; }
  int l; char rest[128];
  if (sscanf(name, "blk.%d.%127s", &l, rest) == 2 && l >= 0 && l < m->c.layers)
    for (int i = 0; i < W_COUNT; i++)
      if (!strcmp(rest, LAYER_NAMES[i])) { free_tensor(&m->layer[l * W_COUNT + i]); m->layer[l * W_COUNT + i] = t; return 0; }
  free(t.vec);
  return -1;
}

or_state *or_state_create(const or_model *m, int context) {
  or_state *s = (or_state *)calloc(1, sizeof(or_state));
  s->context = context;
  s->k = (double **)calloc(m->c.layers, sizeof(double *));
  s->v = (double **)calloc(m->c.layers, sizeof(double *));
  size_t per = (size_t)context * m->c.kv_heads * m->c.head_dim;
  for (int l = 0; l < m->c.layers; l++) { s->k[l] = (double *)calloc(per, sizeof(double)); s->v[l] = (double *)calloc(per, sizeof(double)); }
  return s;
}
/* Benchmark support, not a parity path: fills the K/V rows of positions [0, n) of every
 * layer with deterministic values in [-1, 1), so that a decode can start at position n
 * with the same attention work as after an n-token prompt (the CPU-baseline timing of
 * decode steps deep in the context). Returns 0, or -1 when n exceeds the context. */
int or_state_fill(const or_model *m, or_state *s, int n, uint64_t seed) {
  if (n < 0 || n > s->context) return -1;
  size_t per = (size_t)n * m->c.kv_heads * m->c.head_dim;
  for (int l = 0; l < m->c.layers; l++)
    for (size_t i = 0; i < per; i++) {
      uint64_t z = seed + 0x9e3779b97f4a7c15ull * (i + 1 + (uint64_t)l * per * 2);
      z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
      z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
      z ^= z >> 31;
      s->k[l][i] = (double)(z >> 11) * 0x1.0p-52 - 1.0;
      s->v[l][i] = (double)((z * 0x2545f4914f6cdd1dull) >> 11) * 0x1.0p-52 - 1.0;
    }
  return 0;
}

void or_state_destroy(or_state *s, const or_model *m) {
  if (!s) return;
  for (int l = 0; l < m->c.layers; l++) { free(s->k[l]); free(s->v[l]); }
  free(s->k); free(s->v); free(s);
}

/* verify-dense.mjs:139-143 */
static void rms(const double *x, const double *w, int n, double eps, double *y) {
  double sum = 0;
  for (int i = 0; i < n; i++) sum += x[i] * x[i];
  double inv = 1.0 / sqrt(sum / n + eps);
  for (int i = 0; i < n; i++) y[i] = x[i] * inv * w[i];
}

/* verify-dense.mjs:144-148: out[r] = sum_c x[c] * W[r][c] (+ bias), f64, column order.
 * Rows are independent, so they are spread over threads without changing any value. */
static void project(const double *x, const or_tensor *w, const or_tensor *bias, double *out) {
  int64_t cols = w->cols, rows = w->rows, rb = or_row_bytes(w->type, cols);
#pragma omp parallel num_threads(g_threads)
  {
    double *buf = (double *)malloc(sizeof(double) * cols);
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
      dequant_row(w->data + r * rb, w->type, cols, buf);
      double sum = 0;
      for (int64_t c = 0; c < cols; c++) sum += x[c] * buf[c];
      out[r] = sum + (bias && bias->vec ? bias->vec[r] : 0.0);
    }
    free(buf);
  }
}

static double silu(double g) { return g / (1.0 + exp(-g)); }
/* shaders.ts:136 */
static double gelu_tanh(double x) { return 0.5 * x * (1.0 + tanh(0.7978845608 * (x + 0.044715 * x * x * x))); }

/* One decoder step per token, as verify-dense.mjs:165-211 does; prefill batches
 * are mathematically identical to this token-by-token order (causal attention
 * over the same cached keys). `logits` receives the vocab logits of the LAST id
 * (engine.ts:177-178). Returns 0, or -1 on a bad argument. */
int or_forward(const or_model *m, or_state *s, const int32_t *ids, int n, int start, double *logits) {
  const or_config *c = &m->c;
  int H = c->hidden, heads = c->heads, kvh = c->kv_heads, hd = c->head_dim, group = heads / kvh;
  int qd = heads * hd, kd = kvh * hd, F = c->intermediate;
  if (n < 1 || start < 0 || start + n > s->context) return -1;
  double *x = (double *)malloc(sizeof(double) * H), *normed = (double *)malloc(sizeof(double) * H);
  double *q = (double *)malloc(sizeof(double) * qd), *k = (double *)malloc(sizeof(double) * kd);
  double *v = (double *)malloc(sizeof(double) * kd), *att = (double *)malloc(sizeof(double) * qd);
  double *proj = (double *)malloc(sizeof(double) * H), *gate = (double *)malloc(sizeof(double) * F);
  double *up = (double *)malloc(sizeof(double) * F), *down = (double *)malloc(sizeof(double) * H);
  double *scores = (double *)malloc(sizeof(double) * s->context);
  double *emb = (double *)malloc(sizeof(double) * H);
  int64_t erb = or_row_bytes(m->embd.type, H);
  for (int t = 0; t < n; t++) {
    int pos = start + t;
    if (ids[t] < 0 || ids[t] >= c->vocab) { pos = -1; }
    if (pos < 0) { free(x); free(normed); free(q); free(k); free(v); free(att); free(proj); free(gate); free(up); free(down); free(scores); free(emb); return -1; }
    /* engine.ts:140-144: decoded embedding row, Gemma scales by sqrt(hidden); stored as f32. */
    dequant_row(m->embd.data + (int64_t)ids[t] * erb, m->embd.type, H, emb);
    for (int i = 0; i < H; i++) x[i] = (double)(float)(emb[i] * (c->family == 1 ? sqrt((double)H) : 1.0));
    for (int l = 0; l < c->layers; l++) {
      const or_tensor *L = m->layer + (int64_t)l * W_COUNT;
      int local = c->family == 1 && c->period > 1 && l % c->period != c->period - 1;
      double theta = local ? c->local_theta : c->theta, rscale = local ? 1.0 : c->rope_scale;
      int window = c->family == 1 ? (local ? c->window : s->context) : (c->sliding_window > 0 ? c->sliding_window : s->context);
      rms(x, L[W_ATTN_NORM].vec, H, c->epsilon, normed);
      int dense = c->family == 0;
      project(normed, &L[W_Q], dense && c->bias_q ? &L[W_QB] : NULL, q);
      project(normed, &L[W_K], dense && c->bias_k ? &L[W_KB] : NULL, k);
      project(normed, &L[W_V], dense && c->bias_v ? &L[W_VB] : NULL, v);
      int qkn = c->family == 1 || c->qk_norm;
      int rot = c->family == 1 ? hd : c->rotary_dim;
      for (int h = 0; h < heads; h++) {
        if (qkn) rms_head(q + h * hd, L[W_QN].vec, hd, c->epsilon);
        rotate_head(q + h * hd, hd, rot, qkn ? 0 : c->rope_mode, (double)pos, rscale, theta);
      }
      for (int h = 0; h < kvh; h++) {
        if (qkn) rms_head(k + h * hd, L[W_KN].vec, hd, c->epsilon);
        rotate_head(k + h * hd, hd, rot, qkn ? 0 : c->rope_mode, (double)pos, rscale, theta);
      }
      memcpy(s->k[l] + (int64_t)pos * kd, k, sizeof(double) * kd);
      memcpy(s->v[l] + (int64_t)pos * kd, v, sizeof(double) * kd);
      int end = pos + 1, begin = end - (end < window ? end : window);
      for (int h = 0; h < heads; h++) {
        int kh = h / group;
        double maximum = -INFINITY;
        for (int p = begin; p < end; p++) {
          const double *kv = s->k[l] + (int64_t)p * kd + kh * hd;
          double dot = 0;
          for (int d = 0; d < hd; d++) dot += q[h * hd + d] * kv[d];
          scores[p - begin] = dot * c->attention_scale;
          if (scores[p - begin] > maximum) maximum = scores[p - begin];
        }
        double total = 0;
        for (int p = begin; p < end; p++) { scores[p - begin] = exp(scores[p - begin] - maximum); total += scores[p - begin]; }
        for (int d = 0; d < hd; d++) {
          double sum = 0;
          for (int p = begin; p < end; p++) sum += (scores[p - begin] / total) * s->v[l][(int64_t)p * kd + kh * hd + d];
          att[h * hd + d] = sum;
        }
      }
      project(att, &L[W_O], dense && c->bias_output ? &L[W_OB] : NULL, proj);
      if (!dense) { rms(proj, L[W_POST_ATTN].vec, H, c->epsilon, normed); for (int i = 0; i < H; i++) x[i] += normed[i]; }
      else for (int i = 0; i < H; i++) x[i] += proj[i];
      rms(x, L[W_FFN_NORM].vec, H, c->epsilon, normed);
      if (!dense || c->ffn_gate) {
        project(normed, &L[W_GATE], NULL, gate);
        project(normed, &L[W_UP], NULL, up);
        for (int i = 0; i < F; i++) gate[i] = (c->activation == 1 ? gelu_tanh(gate[i]) : silu(gate[i])) * up[i];
      } else {
        project(normed, &L[W_UP], NULL, gate);
        for (int i = 0; i < F; i++) gate[i] = silu(gate[i]);
      }
      project(gate, &L[W_DOWN], NULL, down);
      if (!dense) { rms(down, L[W_POST_FFW].vec, H, c->epsilon, normed); for (int i = 0; i < H; i++) x[i] += normed[i]; }
      else for (int i = 0; i < H; i++) x[i] += down[i];
    }
    if (t == n - 1 && logits) {
      rms(x, m->out_norm.vec, H, c->epsilon, normed);
      project(normed, m->output.data ? &m->output : &m->embd, NULL, logits);
    }
  }
  free(x); free(normed); free(q); free(k); free(v); free(att); free(proj); free(gate); free(up); free(down); free(scores); free(emb);
  return 0;
}
