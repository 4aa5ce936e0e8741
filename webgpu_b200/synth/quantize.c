/*
 * Seeded synthetic weights in GGML block layouts.
 *
 * The benchmark configurations use random-init models of real architectures, so
 * every weight byte is produced here: N(mean, std) values from a counter-based
 * generator (the value at index i depends only on seed, stream and i, so any
 * thread count gives the same bytes), quantised by block packers written from
 * the layouts that the reference decodes (src/core/quant.ts:11-27 of the
 * reference project). The packers use a plain min/max fit per block; they do
 * not try to minimise quantisation error, and they need not: the decoder and
 * the oracle both read the same bytes.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14 };

/* Worker threads of the OpenMP loops below (a launcher may have set OMP_NUM_THREADS=1). */
void synth_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

static inline uint64_t mix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}
static inline uint64_t draw(uint64_t seed, uint64_t stream, uint64_t i) {
  return mix64(mix64(seed * 0x2545f4914f6cdd1dull + stream) ^ (i * 0xd1342543de82ef95ull));
}
/* Uniform in (0, 1). */
static inline double uniform(uint64_t seed, uint64_t stream, uint64_t i) {
  return ((double)(draw(seed, stream, i) >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}
double synth_uniform(uint64_t seed, uint64_t stream, uint64_t i) { return uniform(seed, stream, i); }
/* Standard normal by Box-Muller over two uniforms of the same counter. */
double synth_normal(uint64_t seed, uint64_t stream, uint64_t i) {
  double u1 = uniform(seed, stream, 2 * i), u2 = uniform(seed, stream, 2 * i + 1);
  return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}
void synth_fill_normal(float *out, int64_t n, uint64_t seed, uint64_t stream, double mean, double std) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; i++) out[i] = (float)(mean + std * synth_normal(seed, stream, (uint64_t)i));
}
/* Integers uniform in [0, n). */
void synth_fill_ints(int32_t *out, int64_t count, uint64_t seed, uint64_t stream, int32_t n) {
  for (int64_t i = 0; i < count; i++) out[i] = (int32_t)(uniform(seed, stream, (uint64_t)i) * n);
}

static inline uint16_t to_half(float f) { _Float16 h = (_Float16)f; uint16_t u; memcpy(&u, &h, 2); return u; }
static inline float from_half(uint16_t u) { _Float16 h; memcpy(&h, &u, 2); return (float)h; }
static inline void put16(uint8_t *p, uint16_t v) { p[0] = v & 255; p[1] = v >> 8; }
static inline int clampi(int v, int lo, int hi) { return v < lo ? lo : v > hi ? hi : v; }

int64_t synth_block_elems(int type) { return type == T_F32 || type == T_F16 ? 1 : type == T_Q4_0 || type == T_Q8_0 ? 32 : 256; }
int64_t synth_block_bytes(int type) {
  switch (type) { case T_F32: return 4; case T_F16: return 2; case T_Q4_0: return 18; case T_Q8_0: return 34;
                  case T_Q4_K: return 144; case T_Q5_K: return 176; case T_Q6_K: return 210; default: return 0; }
}

/* Q4_K / Q5_K super-block: 8 sub-blocks of 32 values, affine q*d*sc - dmin*mn. */
static void pack_kq(const float *x, uint8_t *out, int bits) {
  int levels = (1 << bits) - 1;
  float scale[8], minv[8], maxscale = 0, maxmin = 0;
  for (int s = 0; s < 8; s++) {
    float lo = 0, hi = -INFINITY;
    for (int i = 0; i < 32; i++) { float v = x[32 * s + i]; if (v < lo) lo = v; if (v > hi) hi = v; }
    if (hi < lo) hi = lo;
    scale[s] = (hi - lo) / levels; minv[s] = -lo;
    if (scale[s] > maxscale) maxscale = scale[s];
    if (minv[s] > maxmin) maxmin = minv[s];
  }
  uint16_t dh = to_half(maxscale / 63.0f), mh = to_half(maxmin / 63.0f);
  float d = from_half(dh), dmin = from_half(mh);
  int sc[8], mn[8];
  for (int s = 0; s < 8; s++) {
    sc[s] = d > 0 ? clampi((int)lrintf(scale[s] / d), 0, 63) : 0;
    mn[s] = dmin > 0 ? clampi((int)lrintf(minv[s] / dmin), 0, 63) : 0;
  }
  memset(out, 0, bits == 4 ? 144 : 176);
  put16(out, dh); put16(out + 2, mh);
  uint8_t *S = out + 4;
  for (int s = 0; s < 4; s++) {
    S[s] = (uint8_t)((sc[s] & 63) | ((sc[s + 4] >> 4) << 6));
    S[4 + s] = (uint8_t)((mn[s] & 63) | ((mn[s + 4] >> 4) << 6));
    S[8 + s] = (uint8_t)((sc[s + 4] & 15) | ((mn[s + 4] & 15) << 4));
  }
  uint8_t *qs = out + (bits == 4 ? 16 : 48), *qh = out + 16;
  for (int j = 0; j < 256; j++) {
    int s = j / 32;
    float step = d * sc[s];
    int q = step > 0 ? clampi((int)lrintf((x[j] + dmin * mn[s]) / step), 0, levels) : 0;
    qs[(j / 64) * 32 + j % 32] |= (uint8_t)((q & 15) << ((s % 2) * 4));
    if (bits == 5) qh[j % 32] |= (uint8_t)(((q >> 4) & 1) << s);
  }
}

/* Q6_K super-block: 16 sub-blocks of 16, signed int8 scales, q in [0,63] offset 32. */
static void pack_q6k(const float *x, uint8_t *out) {
  float scale[16], maxscale = 0;
  for (int s = 0; s < 16; s++) {
    float amax = 0;
    for (int i = 0; i < 16; i++) { float a = fabsf(x[16 * s + i]); if (a > amax) amax = a; }
    scale[s] = amax / 31.0f;
    if (scale[s] > maxscale) maxscale = scale[s];
  }
  uint16_t dh = to_half(maxscale / 127.0f);
  float d = from_half(dh);
  memset(out, 0, 210);
  int sc[16];
  for (int s = 0; s < 16; s++) { sc[s] = d > 0 ? clampi((int)lrintf(scale[s] / d), -128, 127) : 0; out[192 + s] = (uint8_t)(int8_t)sc[s]; }
  for (int j = 0; j < 256; j++) {
    int segment = j / 128, quarter = (j % 128) / 32, lane = j % 32, s = j / 16;
    float step = d * sc[s];
    int q = step != 0 ? clampi((int)lrintf(x[j] / step) + 32, 0, 63) : 32;
    out[segment * 64 + (quarter % 2) * 32 + lane] |= (uint8_t)((q & 15) << ((quarter / 2) * 4));
    out[128 + segment * 32 + lane] |= (uint8_t)((q >> 4) << (quarter * 2));
  }
  put16(out + 208, dh);
}

static void pack_q8_0(const float *x, uint8_t *out) {
  float amax = 0;
  for (int i = 0; i < 32; i++) { float a = fabsf(x[i]); if (a > amax) amax = a; }
  uint16_t dh = to_half(amax / 127.0f);
  float d = from_half(dh);
  put16(out, dh);
  for (int i = 0; i < 32; i++) out[2 + i] = (uint8_t)(int8_t)(d > 0 ? clampi((int)lrintf(x[i] / d), -127, 127) : 0);
}

static void pack_q4_0(const float *x, uint8_t *out) {
  float amax = 0;
  for (int i = 0; i < 32; i++) { float a = fabsf(x[i]); if (a > amax) amax = a; }
  uint16_t dh = to_half(amax / 7.0f);
  float d = from_half(dh);
  put16(out, dh);
  memset(out + 2, 0, 16);
  for (int j = 0; j < 32; j++) {
    int q = d > 0 ? clampi((int)lrintf(x[j] / d) + 8, 0, 15) : 8;
    out[2 + j % 16] |= (uint8_t)(q << (j < 16 ? 0 : 4));
  }
}

/* Quantises `rows` rows of `cols` floats into GGUF bytes; returns bytes written or -1. */
int64_t synth_quantize(int type, const float *x, int64_t rows, int64_t cols, uint8_t *out) {
  int64_t be = synth_block_elems(type), bb = synth_block_bytes(type);
  if (!bb || cols % be) return -1;
  int64_t nb = rows * (cols / be);
#pragma omp parallel for schedule(static)
  for (int64_t k = 0; k < nb; k++) {
    const float *src = x + k * be;
    uint8_t *dst = out + k * bb;
    switch (type) {
      case T_F32: memcpy(dst, src, 4); break;
      case T_F16: put16(dst, to_half(src[0])); break;
      case T_Q4_0: pack_q4_0(src, dst); break;
      case T_Q8_0: pack_q8_0(src, dst); break;
      case T_Q4_K: pack_kq(src, dst, 4); break;
      case T_Q5_K: pack_kq(src, dst, 5); break;
      case T_Q6_K: pack_q6k(src, dst); break;
    }
  }
  return nb * bb;
}

/* N(mean, std) values generated and quantised block by block, without holding the
 * float tensor: block k covers value indices [k*be, (k+1)*be) of the row-major
 * tensor. Returns bytes written or -1. */
int64_t synth_normal_quantized(int type, int64_t rows, int64_t cols, uint64_t seed, uint64_t stream,
                               double mean, double std, uint8_t *out) {
  int64_t be = synth_block_elems(type), bb = synth_block_bytes(type);
  if (!bb || cols % be) return -1;
  int64_t nb = rows * (cols / be);
  if (type == T_F32 || type == T_F16) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < nb; i++) {
      float v = (float)(mean + std * synth_normal(seed, stream, (uint64_t)i));
      if (type == T_F32) memcpy(out + 4 * i, &v, 4); else put16(out + 2 * i, to_half(v));
    }
    return nb * bb;
  }
#pragma omp parallel for schedule(static)
  for (int64_t k = 0; k < nb; k++) {
    float buf[256];
    for (int64_t i = 0; i < be; i++) buf[i] = (float)(mean + std * synth_normal(seed, stream, (uint64_t)(k * be + i)));
    uint8_t *dst = out + k * bb;
    switch (type) {
      case T_Q4_0: pack_q4_0(buf, dst); break;
      case T_Q8_0: pack_q8_0(buf, dst); break;
      case T_Q4_K: pack_kq(buf, dst, 4); break;
      case T_Q5_K: pack_kq(buf, dst, 5); break;
      case T_Q6_K: pack_q6k(buf, dst); break;
    }
  }
  return nb * bb;
}

/* GEMV microbench blocks: every byte uniform, then the fp16 scale fields replaced by
 * |N(0, scale_std)| (Q4_K d and dmin; Q6_K d) and, for Q6_K, the int8 scales drawn
 * uniform in [-32, 31]. */
int64_t synth_random_blocks(int type, int64_t nblocks, uint64_t seed, uint64_t stream, double scale_std, uint8_t *out) {
  int64_t bb = synth_block_bytes(type);
  if (!bb) return -1;
#pragma omp parallel for schedule(static)
  for (int64_t k = 0; k < nblocks; k++) {
    uint8_t *dst = out + k * bb;
    for (int64_t i = 0; i < bb; i++) dst[i] = (uint8_t)(draw(seed, stream, (uint64_t)(k * bb + i)) >> 56);
    uint64_t base = (uint64_t)nblocks * bb + (uint64_t)k * 32;
    if (type == T_Q4_K || type == T_Q5_K) {
      put16(dst, to_half((float)fabs(scale_std * synth_normal(seed, stream, base))));
      put16(dst + 2, to_half((float)fabs(scale_std * synth_normal(seed, stream, base + 1))));
    } else if (type == T_Q6_K) {
      for (int s = 0; s < 16; s++) dst[192 + s] = (uint8_t)(int8_t)((int)(uniform(seed, stream, 2 * (base + 2 + s)) * 64) - 32);
      put16(dst + 208, to_half((float)fabs(scale_std * synth_normal(seed, stream, base))));
    } else if (type == T_Q4_0 || type == T_Q8_0) {
      put16(dst, to_half((float)fabs(scale_std * synth_normal(seed, stream, base))));
    } else if (type == T_F16) {
      put16(dst, to_half((float)(synth_normal(seed, stream, base))));
    } else if (type == T_F32) {
      float v = (float)synth_normal(seed, stream, base); memcpy(dst, &v, 4);
    }
  }
  return nblocks * bb;
}
