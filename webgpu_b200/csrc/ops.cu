// Decoder block kernels other than the GEMV: layout repack, dequant, embedding
// gather, RMSNorm, fused Q/K-norm + RoPE + KV ring write, split-K attention
// with in-kernel merge, argmax. Reference shaders (src/core/shaders.ts of the
// reference project): normShader :84-97, ropeShader :98-116, attentionShader
// :117-150, addShader :152-157, ropeNeoxShader :168-181, ropeClassicShader
// :184-197; greedy sample engine.ts:305-309; embedding engine.ts:140-144.
#include <float.h>
#include "kernels.h"
#include "quant.cuh"
#include "tile.cuh"

namespace wgd {

// ------------------------------------------------------------------ repack

__device__ __forceinline__ int map_row(const RowMap &m, int grow) {
  int i = grow - m.src_begin;
  if (m.interleave == 0) return m.dst_base + i;
  const int R = m.glu_block;
  return (i / R) * 2 * R + (m.interleave == 2 ? R : 0) + (i % R);
}

__global__ void repack_kernel(int type, const uint8_t *src, int64_t srb, int row0, int nrows, int blk0, int nbl, uint8_t *dst,
                              int64_t drb, RowMap m) {
  const int bb = type == F32 ? 4 : type == F16 ? 2 : type == Q4_0 ? 18 : type == Q8_0 ? 34 : type == Q4_K ? 144 : type == Q5_K ? 176 : 210;
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)nrows * nbl) return;
  int r = (int)(idx / nbl), bi = (int)(idx % nbl);
  int grow = row0 + r;
  if (grow < m.src_begin || grow >= m.src_end) return;
  int drow = map_row(m, grow);
  repack_block(type, src + (int64_t)r * srb + (int64_t)(blk0 + bi) * bb, dst + (int64_t)drow * drb, bi, nbl);
}

cudaError_t launch_repack(int type, const uint8_t *src, int64_t src_row_bytes, int row0, int nrows, int blk0, int nbl,
                          uint8_t *dst, int64_t dst_row_bytes, RowMap map, cudaStream_t s) {
  int64_t total = (int64_t)nrows * nbl;
  if (total == 0) return cudaSuccess;
  int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  repack_kernel<<<(unsigned)blocks, threads, 0, s>>>(type, src, src_row_bytes, row0, nrows, blk0, nbl, dst, dst_row_bytes, map);
  return cudaGetLastError();
}

__global__ void repack_tiled_kernel(int type, const uint8_t *src, int64_t srb, int row0, int nrows, int blk0, int nbl, uint8_t *dst,
                                    RowMap m) {
  const int bb = type == Q4_K ? 144 : 210;
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)nrows * nbl) return;
  int r = (int)(idx / nbl), bi = (int)(idx % nbl);
  int grow = row0 + r;
  if (grow < m.src_begin || grow >= m.src_end) return;
  const int drow = map_row(m, grow), t = drow >> 4, lr = drow & 15;
  const uint8_t *s = src + (int64_t)r * srb + (int64_t)(blk0 + bi) * bb;
  uint8_t *chunk = dst + ((int64_t)t * nbl + bi) * (16 * bb);
  for (int b = 0; b < bb; b++) chunk[tile_offset(type, lr, b)] = s[b];
}

cudaError_t launch_repack_tiled(int type, const uint8_t *src, int64_t src_row_bytes, int row0, int nrows, int blk0, int nbl,
                                uint8_t *dst, int dst_rows, RowMap map, cudaStream_t s) {
  (void)dst_rows;
  if (!tiled_type(type)) return cudaErrorInvalidValue;
  int64_t total = (int64_t)nrows * nbl;
  if (total == 0) return cudaSuccess;
  repack_tiled_kernel<<<(unsigned)((total + 127) / 128), 128, 0, s>>>(type, src, src_row_bytes, row0, nrows, blk0, nbl, dst, map);
  return cudaGetLastError();
}

template <int T>
__global__ void dequant_tiled_kernel(const uint8_t *w, int rows, int cols, float *out, int64_t ldo) {
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)rows * cols) return;
  int r = (int)(idx / cols), c = (int)(idx % cols);
  out[(int64_t)r * ldo + c] = dequant_tiled<T>(w, cols / 256, r, c);
}

cudaError_t launch_dequant_tiled(int type, const uint8_t *w, int rows, int cols, float *out, int64_t ldo, cudaStream_t s) {
  int64_t total = (int64_t)rows * cols;
  if (total == 0) return cudaSuccess;
  const unsigned blocks = (unsigned)((total + 255) / 256);
  if (type == Q4_K) dequant_tiled_kernel<Q4_K><<<blocks, 256, 0, s>>>(w, rows, cols, out, ldo);
  else if (type == Q6_K) dequant_tiled_kernel<Q6_K><<<blocks, 256, 0, s>>>(w, rows, cols, out, ldo);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

// ------------------------------------------------------------------ dequant

template <int T>
__global__ void dequant_kernel(const uint8_t *w, int64_t drow, int rows, int cols, float *out, int64_t ldo) {
  const int nb = cols / block_elems_dev<T>();
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)rows * cols) return;
  int r = (int)(idx / cols), c = (int)(idx % cols);
  out[(int64_t)r * ldo + c] = dequant_elem<T>(w + (int64_t)r * drow, nb, c);
}

template <int T>
static cudaError_t dq(const uint8_t *w, int64_t drow, int rows, int cols, float *out, int64_t ldo, cudaStream_t s) {
  int64_t total = (int64_t)rows * cols;
  if (total == 0) return cudaSuccess;
  dequant_kernel<T><<<(unsigned)((total + 255) / 256), 256, 0, s>>>(w, drow, rows, cols, out, ldo);
  return cudaGetLastError();
}

cudaError_t launch_dequant(int type, const uint8_t *w, int64_t drow, int rows, int cols, float *out, int64_t ldo, cudaStream_t s) {
  switch (type) {
    case F32: return dq<F32>(w, drow, rows, cols, out, ldo, s);
    case F16: return dq<F16>(w, drow, rows, cols, out, ldo, s);
    case Q4_0: return dq<Q4_0>(w, drow, rows, cols, out, ldo, s);
    case Q8_0: return dq<Q8_0>(w, drow, rows, cols, out, ldo, s);
    case Q4_K: return dq<Q4_K>(w, drow, rows, cols, out, ldo, s);
    case Q5_K: return dq<Q5_K>(w, drow, rows, cols, out, ldo, s);
    case Q6_K: return dq<Q6_K>(w, drow, rows, cols, out, ldo, s);
    default: return cudaErrorInvalidValue;
  }
}

// ------------------------------------------------------------------ embed

template <int T>
__global__ void embed_kernel(const uint8_t *w, int64_t drow, int cols, const int *ids, int vocab, float scale, float *out,
                             int ldo, int *err) {
  pdl_wait();
  const int t = blockIdx.x, nb = cols / block_elems_dev<T>();
  const int id = ids[t];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && threadIdx.x == 0 && err) *err = 1;
  for (int c = threadIdx.x; c < cols; c += blockDim.x)
    out[(int64_t)t * ldo + c] = ok ? dequant_elem<T>(w + (int64_t)id * drow, nb, c) * scale : 0.f;
  pdl_launch_dependents();
}

template <int T>
__global__ void embed_tiled_kernel(const uint8_t *w, int cols, const int *ids, int vocab, float scale, float *out, int ldo, int *err) {
  pdl_wait();
  const int t = blockIdx.x;
  const int id = ids[t];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && threadIdx.x == 0 && err) *err = 1;
  for (int c = threadIdx.x; c < cols; c += blockDim.x)
    out[(int64_t)t * ldo + c] = ok ? dequant_tiled<T>(w, cols / 256, id, c) * scale : 0.f;
  pdl_launch_dependents();
}

template <int T>
static cudaError_t emb(const uint8_t *w, int64_t drow, int cols, const int *ids, int n, int vocab, float scale, float *out,
                       int ldo, int *err, cudaStream_t s, bool pdl) {
  return launch_k(embed_kernel<T>, dim3(n), dim3(256), 0, s, pdl, w, drow, cols, ids, vocab, scale, out, ldo, err);
}

cudaError_t launch_embed(int type, const uint8_t *w, int64_t drow, int cols, const int *ids, int n, int vocab, float scale,
                         float *out, int ldo, int *err, cudaStream_t s, bool pdl, bool tiled) {
  if (tiled) {
    if (type == Q4_K) return launch_k(embed_tiled_kernel<Q4_K>, dim3(n), dim3(256), 0, s, pdl, w, cols, ids, vocab, scale, out, ldo, err);
    if (type == Q6_K) return launch_k(embed_tiled_kernel<Q6_K>, dim3(n), dim3(256), 0, s, pdl, w, cols, ids, vocab, scale, out, ldo, err);
    return cudaErrorInvalidValue;
  }
  switch (type) {
    case F32: return emb<F32>(w, drow, cols, ids, n, vocab, scale, out, ldo, err, s, pdl);
    case F16: return emb<F16>(w, drow, cols, ids, n, vocab, scale, out, ldo, err, s, pdl);
    case Q4_0: return emb<Q4_0>(w, drow, cols, ids, n, vocab, scale, out, ldo, err, s, pdl);
    case Q8_0: return emb<Q8_0>(w, drow, cols, ids, n, vocab, scale, out, ldo, err, s, pdl);
    case Q4_K: return emb<Q4_K>(w, drow, cols, ids, n, vocab, scale, out, ldo, err, s, pdl);
    case Q5_K: return emb<Q5_K>(w, drow, cols, ids, n, vocab, scale, out, ldo, err, s, pdl);
    case Q6_K: return emb<Q6_K>(w, drow, cols, ids, n, vocab, scale, out, ldo, err, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

// ------------------------------------------------------------------ rmsnorm

__device__ __forceinline__ float block_sum(float v, float *sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < nw; w++) t += sh[w];
  return t;
}

__global__ void rmsnorm_kernel(const float *x, int ldx, const float *w, float eps, int cols, float *y, int ldy, int add) {
  __shared__ float sh[32];
  pdl_wait();
  const float *xr = x + (int64_t)blockIdx.x * ldx;
  float *yr = y + (int64_t)blockIdx.x * ldy;
  float s = 0.f;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) s = fmaf(xr[c], xr[c], s);
  const float inv = rsqrtf(block_sum(s, sh) / (float)cols + eps);
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    const float v = xr[c] * inv * w[c];
    if (add) yr[c] += v; else yr[c] = v;
  }
  pdl_launch_dependents();
}

cudaError_t launch_rmsnorm(const float *x, int ldx, const float *w, float eps, int cols, int n, float *y, int ldy, int add,
                           cudaStream_t s, bool pdl) {
  if (n <= 0) return cudaSuccess;
  return launch_k(rmsnorm_kernel, dim3(n), dim3(512), 0, s, pdl, x, ldx, w, eps, cols, y, ldy, add);
}

// ------------------------------------------------------------ rope + kv write

// One CTA per (row t, head). Heads [0, heads) are query heads (written to
// q_out); heads [heads, heads+kv_heads) are key heads, whose rotated vector and
// the matching value head are written into ring slot (start+t) % capacity.
// The angle is computed in double: (start+t) * scale / theta^(2i/rot).
__global__ void rope_kv_kernel(const RopeArgs a) {
  extern __shared__ float hv[];  // [hd]
  __shared__ float sh[32];
  pdl_wait();
  const int t = blockIdx.x, h = blockIdx.y, hd = a.hd;
  const int start = a.start ? *a.start : a.start_host;
  const int pos = start + t;
  const bool is_q = h < a.heads;
  const int kh = h - a.heads;
  const float *src = a.qkv + (int64_t)t * a.ld + (int64_t)h * hd;
  const float *nw = is_q ? a.q_norm : a.k_norm;
  for (int d = threadIdx.x; d < hd; d += blockDim.x) hv[d] = src[d];
  __syncthreads();
  if (nw) {
    float s = 0.f;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) s = fmaf(hv[d], hv[d], s);
    const float inv = rsqrtf(block_sum(s, sh) / (float)hd + a.eps);
    __syncthreads();
    for (int d = threadIdx.x; d < hd; d += blockDim.x) hv[d] = hv[d] * inv * nw[d];
    __syncthreads();
  }
  const int rot = a.rot, half = rot / 2;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const double angle = (double)pos * a.scale / pow(a.theta, (2.0 * i) / rot);
    double sn, cs;
    sincos(angle, &sn, &cs);
    const float c = (float)cs, s = (float)sn;
    const int ia = a.mode == 0 ? i : 2 * i, ib = a.mode == 0 ? i + half : 2 * i + 1;
    const float l = hv[ia], r = hv[ib];
    hv[ia] = l * c - r * s;
    hv[ib] = l * s + r * c;
  }
  __syncthreads();
  if (is_q) {
    float *dst = a.q_out + ((int64_t)t * a.heads + h) * hd;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) dst[d] = hv[d];
  } else {
    const int slot = pos % a.capacity;
    float *kd = a.k_cache + ((int64_t)kh * a.capacity + slot) * hd;
    float *vd = a.v_cache + ((int64_t)kh * a.capacity + slot) * hd;
    const float *vs = a.qkv + (int64_t)t * a.ld + (int64_t)(a.heads + a.kv_heads + kh) * hd;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) { kd[d] = hv[d]; vd[d] = vs[d]; }
  }
  pdl_launch_dependents();
}

cudaError_t launch_rope_kv(const RopeArgs &a, cudaStream_t s, bool pdl) {
  if (a.n <= 0) return cudaSuccess;
  int threads = a.hd >= 128 ? 128 : (a.hd < 32 ? 32 : a.hd);
  return launch_k(rope_kv_kernel, dim3(a.n, a.heads + a.kv_heads), dim3(threads), a.hd * sizeof(float), s, pdl, a);
}

// ------------------------------------------------------------------ attention

// Split-K decode attention with an in-kernel merge (flash-decoding). CTA
// (t*kv_heads + kh, sp) scores keys [p0, p1) of query row t against all G =
// heads/kv_heads query heads of KV head kh, keeps an online softmax (max, sum,
// weighted V) over 128-key tiles, and writes a partial; the last CTA of the
// (t, kh) pair merges the partials in split order. Keys are read from ring slot
// p % capacity of the [kv_heads][capacity][hd] cache (attentionShader
// semantics: window [end - min(end, window), end), end = start + t + 1).
constexpr int ATT_THREADS = 128, ATT_TILE = 128, ATT_GMAX = 8, ATT_MINCHUNK = 64, ATT_MAXSPLIT = 64;

int attention_splits(int max_len) {
  int s = (max_len + ATT_MINCHUNK - 1) / ATT_MINCHUNK;
  return s < 1 ? 1 : s > ATT_MAXSPLIT ? ATT_MAXSPLIT : s;
}
size_t attention_part_floats(int n, int heads, int kv_heads, int hd, int splits) {
  return (size_t)n * kv_heads * splits * (heads / kv_heads) * (hd + 2);
}

__global__ void __launch_bounds__(ATT_THREADS) attention_kernel(const AttnArgs a) {
  extern __shared__ float sm[];
  const int G = a.heads / a.kv_heads, hd = a.hd;
  float *q_s = sm;                          // [G][hd]
  float *e_s = q_s + G * hd;                // [G][ATT_TILE]
  float *red = e_s + G * ATT_TILE;          // [G][4] warp partials
  float *acc_s = red + G * 4;               // [G][hd] position-group partials
  __shared__ float m_s[ATT_GMAX], l_s[ATT_GMAX], corr_s[ATT_GMAX];
  __shared__ int last_s;
  pdl_wait();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t = blockIdx.x / a.kv_heads, kh = blockIdx.x % a.kv_heads, sp = blockIdx.y;
  const int start = a.start ? *a.start : a.start_host;
  const int end = start + t + 1, begin = end - (end < a.window ? end : a.window), L = end - begin;
  int chunk = (L + a.splits - 1) / a.splits;
  if (chunk < ATT_MINCHUNK) chunk = ATT_MINCHUNK;
  const int nsp = (L + chunk - 1) / chunk;
  if (sp >= nsp) return;
  const int p0 = begin + sp * chunk, p1 = min(end, p0 + chunk);

  for (int i = tid; i < G * hd; i += ATT_THREADS) q_s[i] = a.q[((int64_t)t * a.heads + kh * G) * hd + i];
  if (tid < G) { m_s[tid] = -FLT_MAX; l_s[tid] = 0.f; }
  // PV mapping: thread handles dims d = dsub + 128k of position group pg.
  const int dlanes = hd < ATT_THREADS ? hd : ATT_THREADS;
  const int pgroups = ATT_THREADS / dlanes;
  const int dsub = tid % dlanes, pg = tid / dlanes;
  const bool pv_live = pg < pgroups;
  float acc[ATT_GMAX][4];
#pragma unroll
  for (int g = 0; g < ATT_GMAX; g++)
#pragma unroll
    for (int k = 0; k < 4; k++) acc[g][k] = 0.f;
  const float *kb = a.k + (int64_t)kh * a.capacity * hd;
  const float *vb = a.v + (int64_t)kh * a.capacity * hd;
  __syncthreads();

  for (int tile = p0; tile < p1; tile += ATT_TILE) {
    const int p = tile + tid;
    const bool live = p < p1;
    float s[ATT_GMAX];
#pragma unroll
    for (int g = 0; g < ATT_GMAX; g++) s[g] = 0.f;
    if (live) {
      const float4 *kr = reinterpret_cast<const float4 *>(kb + (int64_t)(p % a.capacity) * hd);
      for (int d4 = 0; d4 < hd / 4; d4++) {
        const float4 k4 = __ldg(kr + d4);
#pragma unroll
        for (int g = 0; g < ATT_GMAX; g++) {
          if (g < G) {
            const float4 q4 = reinterpret_cast<const float4 *>(q_s + g * hd)[d4];
            s[g] = fmaf(q4.x, k4.x, fmaf(q4.y, k4.y, fmaf(q4.z, k4.z, fmaf(q4.w, k4.w, s[g]))));
          }
        }
      }
    }
    // tile max per head
#pragma unroll
    for (int g = 0; g < ATT_GMAX; g++) {
      if (g < G) {
        s[g] = live ? s[g] * a.scale : -FLT_MAX;
        float mx = warp_max(s[g]);
        if (lane == 0) red[g * 4 + warp] = mx;
      }
    }
    __syncthreads();
    if (tid < G) {
      float mx = fmaxf(fmaxf(red[tid * 4], red[tid * 4 + 1]), fmaxf(red[tid * 4 + 2], red[tid * 4 + 3]));
      float mnew = fmaxf(m_s[tid], mx);
      corr_s[tid] = expf(m_s[tid] - mnew);
      m_s[tid] = mnew;
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < ATT_GMAX; g++) {
      if (g < G) {
        float e = live ? expf(s[g] - m_s[g]) : 0.f;
        e_s[g * ATT_TILE + tid] = e;
        float sum = warp_sum(e);
        if (lane == 0) red[g * 4 + warp] = sum;
      }
    }
    __syncthreads();
    if (tid < G) l_s[tid] = l_s[tid] * corr_s[tid] + ((red[tid * 4] + red[tid * 4 + 1]) + (red[tid * 4 + 2] + red[tid * 4 + 3]));
    // PV over this tile
    const int cnt = min(ATT_TILE, p1 - tile);
#pragma unroll
    for (int g = 0; g < ATT_GMAX; g++)
      if (g < G)
#pragma unroll
        for (int k = 0; k < 4; k++) acc[g][k] *= corr_s[g];
    for (int j = pg; pv_live && j < cnt; j += pgroups) {
      const float *vr = vb + (int64_t)((tile + j) % a.capacity) * hd;
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const int d = dsub + k * ATT_THREADS;
        if (d < hd) {
          const float v = __ldg(vr + d);
#pragma unroll
          for (int g = 0; g < ATT_GMAX; g++)
            if (g < G) acc[g][k] = fmaf(e_s[g * ATT_TILE + j], v, acc[g][k]);
        }
      }
    }
    __syncthreads();
  }
  // combine position groups into acc_s[g][d]
  for (int i = tid; i < G * hd; i += ATT_THREADS) acc_s[i] = 0.f;
  __syncthreads();
  for (int q = 0; q < pgroups; q++) {
    if (pg == q) {
#pragma unroll
      for (int g = 0; g < ATT_GMAX; g++)
        if (g < G)
#pragma unroll
          for (int k = 0; k < 4; k++) {
            const int d = dsub + k * ATT_THREADS;
            if (d < hd) acc_s[g * hd + d] += acc[g][k];
          }
    }
    __syncthreads();
  }
  const int pair = t * a.kv_heads + kh;
  float *out_base = a.out + ((int64_t)t * a.heads + kh * G) * hd;
  if (nsp == 1) {
    for (int i = tid; i < G * hd; i += ATT_THREADS) out_base[i] = acc_s[i] / l_s[i / hd];
    pdl_launch_dependents();
    return;
  }
  float *part = a.part + ((int64_t)pair * a.splits + sp) * G * (hd + 2);
  for (int i = tid; i < G * hd; i += ATT_THREADS) part[(i / hd) * (hd + 2) + 2 + (i % hd)] = acc_s[i];
  if (tid < G) { part[tid * (hd + 2)] = m_s[tid]; part[tid * (hd + 2) + 1] = l_s[tid]; }
  __threadfence();
  __syncthreads();
  if (tid == 0) last_s = atomicAdd(a.ctr + pair, 1u) == (unsigned)(nsp - 1);
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  const float *pb = a.part + (int64_t)pair * a.splits * G * (hd + 2);
  for (int i = tid; i < G * hd; i += ATT_THREADS) {
    const int g = i / hd, d = i % hd;
    float M = -FLT_MAX;
    for (int j = 0; j < nsp; j++) M = fmaxf(M, __ldcg(pb + ((int64_t)j * G + g) * (hd + 2)));
    float num = 0.f, den = 0.f;
    for (int j = 0; j < nsp; j++) {
      const float *pp = pb + ((int64_t)j * G + g) * (hd + 2);
      const float w = expf(__ldcg(pp) - M);
      den = fmaf(w, __ldcg(pp + 1), den);
      num = fmaf(w, __ldcg(pp + 2 + d), num);
    }
    out_base[i] = num / den;
  }
  if (tid == 0) a.ctr[pair] = 0u;
  pdl_launch_dependents();
}

cudaError_t launch_attention(const AttnArgs &a, cudaStream_t s, bool pdl) {
  const int G = a.heads / a.kv_heads;
  if (G > ATT_GMAX || a.hd % 4 || a.hd > 4 * ATT_THREADS || a.splits < 1 || a.splits > ATT_MAXSPLIT) return cudaErrorInvalidValue;
  size_t smem = sizeof(float) * ((size_t)G * a.hd * 2 + (size_t)G * ATT_TILE + G * 4);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    attr = true;
  }
  return launch_k(attention_kernel, dim3(a.n * a.kv_heads, a.splits), dim3(ATT_THREADS), smem, s, pdl, a);
}

// ------------------------------------------------------------------ argmax

constexpr int AM_THREADS = 512, AM_PER_BLOCK = 8192, AM_MAXBLOCKS = 256;
int argmax_blocks(int n) {
  int b = (n + AM_PER_BLOCK - 1) / AM_PER_BLOCK;
  return b < 1 ? 1 : b > AM_MAXBLOCKS ? AM_MAXBLOCKS : b;
}

// (value, index) better: larger finite value, or equal value with smaller index.
__device__ __forceinline__ bool am_better(float v, int i, float bv, int bi) {
  return bi < 0 || v > bv || (v == bv && i < bi);
}
__device__ __forceinline__ void am_block(float &bv, int &bi, float *shv, int *shi) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (oi >= 0 && am_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
  }
  if (lane == 0) { shv[warp] = bv; shi[warp] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); w++)
      if (shi[w] >= 0 && am_better(shv[w], shi[w], bv, bi)) { bv = shv[w]; bi = shi[w]; }
  }
}

__global__ void argmax_kernel(const float *x, int n, int *out_idx, float *out_val, float *part, unsigned *ctr) {
  __shared__ float shv[32];
  __shared__ int shi[32];
  __shared__ int last_s;
  pdl_wait();
  const int per = (n + gridDim.x - 1) / gridDim.x;
  const int lo = blockIdx.x * per, hi = min(n, lo + per);
  float bv = -FLT_MAX;
  int bi = -1;
  for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const float v = x[i];
    if (isfinite(v) && am_better(v, i, bv, bi)) { bv = v; bi = i; }
  }
  am_block(bv, bi, shv, shi);
  if (threadIdx.x == 0) {
    part[2 * blockIdx.x] = bv;
    part[2 * blockIdx.x + 1] = __int_as_float(bi);
    __threadfence();
    last_s = atomicAdd(ctr, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  bv = -FLT_MAX;
  bi = -1;
  for (int b = threadIdx.x; b < (int)gridDim.x; b += blockDim.x) {
    const float v = __ldcg(part + 2 * b);
    const int i = __float_as_int(__ldcg(part + 2 * b + 1));
    if (i >= 0 && am_better(v, i, bv, bi)) { bv = v; bi = i; }
  }
  __syncthreads();
  am_block(bv, bi, shv, shi);
  if (threadIdx.x == 0) {
    *out_idx = bi;
    if (out_val) *out_val = bv;
    *ctr = 0u;
  }
  pdl_launch_dependents();
}

cudaError_t launch_argmax(const float *x, int n, int *out_idx, float *out_val, float *part, unsigned *ctr, cudaStream_t s,
                          bool pdl) {
  return launch_k(argmax_kernel, dim3(argmax_blocks(n)), dim3(AM_THREADS), 0, s, pdl, x, n, out_idx, out_val, part, ctr);
}

// ------------------------------------------------------------------ advance

__global__ void advance_kernel(int *ids, int *start, const int *argmax, int *tokens, int *step, int *err) {
  pdl_wait();
  const int tok = *argmax;
  if (tok < 0) *err = 2;
  ids[0] = tok < 0 ? 0 : tok;
  *start += 1;
  tokens[*step] = tok;
  *step += 1;
  pdl_launch_dependents();
}
cudaError_t launch_advance(int *ids, int *start, const int *argmax, int *tokens, int *step, int *err, cudaStream_t s, bool pdl) {
  return launch_k(advance_kernel, dim3(1), dim3(1), 0, s, pdl, ids, start, argmax, tokens, step, err);
}

// ------------------------------------------------------------------ add

__global__ void add_kernel(const float *x, float *y, int64_t n) {
  pdl_wait();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) y[i] += x[i];
  pdl_launch_dependents();
}
cudaError_t launch_add(const float *x, float *y, int64_t n, cudaStream_t s, bool pdl) {
  if (n <= 0) return cudaSuccess;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  return launch_k(add_kernel, dim3((unsigned)blocks), dim3(256), 0, s, pdl, x, y, n);
}

}  // namespace wgd
