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
    if (add) yr[c] = __ldcg(yr + c) + v; else yr[c] = v;  // residual read through L2
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
    float c, s;
    if (a.table) {
      const float2 cs2 = a.table[(int64_t)pos * half + i];
      c = cs2.x;
      s = cs2.y;
    } else {
      const double angle = (double)pos * a.scale / pow(a.theta, (2.0 * i) / rot);
      double sn, cs;
      sincos(angle, &sn, &cs);
      c = (float)cs;
      s = (float)sn;
    }
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

// Split-K attention with an in-kernel merge (flash-decoding). CTA
// (t*kv_heads + kh, sp) scores keys [p0, p1) of query row t against all G =
// heads/kv_heads query heads of KV head kh and writes a partial (running max,
// sum, weighted V); the last CTA of the (t, kh) pair merges the partials in
// split order. Keys are read from ring slot p % capacity of the
// [kv_heads][capacity][hd] cache (attentionShader semantics: window
// [end - min(end, window), end), end = start + t + 1).
//
// K and V rows are staged 32 at a time into shared memory with cp.async (two
// stages when they fit), rows padded to hd + 4 floats so that lane-per-row
// reads are bank-conflict free. Warp w owns query heads w and w + 4: lane j
// scores key j of the tile, the online softmax lives in registers, and for PV
// lane l accumulates dims [4l, 4l + 4) (+128 per extra float4) of its heads.
constexpr int ATT_THREADS = 128, ATT_WARPS = 4, ATT_TILE = 32, ATT_GMAX = 8, ATT_MAXSPLIT = 64;
constexpr int ATT_CHUNK_DECODE = 32, ATT_CHUNK_ROWS = 64;

int attention_splits(int max_len) {
  int s = (max_len + ATT_CHUNK_DECODE - 1) / ATT_CHUNK_DECODE;
  return s < 1 ? 1 : s > ATT_MAXSPLIT ? ATT_MAXSPLIT : s;
}
size_t attention_part_floats(int n, int heads, int kv_heads, int hd, int splits) {
  return (size_t)n * kv_heads * splits * (heads / kv_heads) * (hd + 4);
}

__device__ __forceinline__ void cp_async16(void *smem, const void *g) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
__device__ __forceinline__ float4 f4_fma(float s, float4 v, float4 a) {
  return make_float4(fmaf(s, v.x, a.x), fmaf(s, v.y, a.y), fmaf(s, v.z, a.z), fmaf(s, v.w, a.w));
}

// NI = float4s per lane per head row (hd <= 128 * NI).
template <int NI>
__global__ void __launch_bounds__(ATT_THREADS) attention_kernel(const AttnArgs a) {
  extern __shared__ __align__(16) float sm[];
  const int G = a.heads / a.kv_heads, hd = a.hd, hd4 = hd >> 2, RS = hd + 4;
  const int nst = hd <= 256 ? 2 : 1;
  float *q_s = sm;              // [G][hd]
  float *kn_s = q_s + G * hd;   // new K row (fused decode)
  float *vn_s = kn_s + hd;      // new V row
  float *kv_s = vn_s + hd;      // [nst][K|V][ATT_TILE][RS]
  __shared__ int last_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t = blockIdx.x / a.kv_heads, kh = blockIdx.x % a.kv_heads, sp = blockIdx.y;
  const bool fused = a.qkv != nullptr;
  // In fused decode mode every cached row but the new one was written by an
  // earlier token's kernels (already complete), and `start` by the previous
  // step's advance kernel, so staging may begin before the dependency wait.
  if (!fused) pdl_wait();
  const int start = a.start ? *a.start : a.start_host;
  const int end = start + t + 1, begin = end - (end < a.window ? end : a.window), L = end - begin;
  const int minc = a.n == 1 ? ATT_CHUNK_DECODE : ATT_CHUNK_ROWS;
  int chunk = (L + a.splits - 1) / a.splits;
  if (chunk < minc) chunk = minc;
  const int nsp = (L + chunk - 1) / chunk;
  if (sp >= nsp) {
    if (fused) pdl_wait();
    return;
  }
  const int p0 = begin + sp * chunk, p1 = min(end, p0 + chunk);
  const bool owns_new = fused && p1 == end;  // this CTA scores the new position
  const float *kb = a.k + (int64_t)kh * a.capacity * hd;
  const float *vb = a.v + (int64_t)kh * a.capacity * hd;
  const int ntiles = (p1 - p0 + ATT_TILE - 1) / ATT_TILE;

  auto stage = [&](int tile, int st) {
    const int cnt = min(ATT_TILE, p1 - tile), total = cnt * hd4;
    float *ks = kv_s + (size_t)st * 2 * ATT_TILE * RS, *vs = ks + ATT_TILE * RS;
    for (int i = tid; i < total; i += ATT_THREADS) {
      const int r = i / hd4, c = (i - r * hd4) * 4;
      const int p = tile + r;
      if (owns_new && p == end - 1) continue;  // filled from shared memory below
      const int64_t row = (int64_t)(p % a.capacity) * hd;
      cp_async16(ks + r * RS + c, kb + row + c);
      cp_async16(vs + r * RS + c, vb + row + c);
    }
    cp_async_commit();
  };
  stage(p0, 0);
  if (nst == 2 && ntiles > 1) stage(p0 + ATT_TILE, 1);

  if (fused) pdl_wait();
  if (!fused) {
    for (int i = tid; i < G * hd; i += ATT_THREADS) q_s[i] = a.q[((int64_t)t * a.heads + kh * G) * hd + i];
  } else {
    const int hq = G + (owns_new ? 1 : 0);  // q heads, then the k head when this CTA owns the new row
    for (int i = tid; i < hq * hd; i += ATT_THREADS) {
      const int g = i / hd, d = i - g * hd;
      const float *src = g < G ? a.qkv + (int64_t)(kh * G + g) * hd : a.qkv + (int64_t)(a.heads + kh) * hd;
      (g < G ? q_s + g * hd : kn_s)[d] = src[d];
    }
    if (owns_new)
      for (int d = tid; d < hd; d += ATT_THREADS) vn_s[d] = a.qkv[(int64_t)(a.heads + a.kv_heads + kh) * hd + d];
    __syncthreads();
    // per-head RMS norm (Q/K norm) then rotation, one warp per head
    for (int g = warp; g < hq; g += ATT_WARPS) {
      float *hv = g < G ? q_s + g * hd : kn_s;
      const float *nw = g < G ? a.q_norm : a.k_norm;
      if (nw) {
        float ss = 0.f;
        for (int d = lane; d < hd; d += 32) ss = fmaf(hv[d], hv[d], ss);
        const float inv = rsqrtf(warp_sum(ss) / (float)hd + a.eps);
        __syncwarp();
        for (int d = lane; d < hd; d += 32) hv[d] = hv[d] * inv * nw[d];
        __syncwarp();
      }
      const int half = a.rot / 2;
      const float2 *tb = a.table + (int64_t)start * half;
      for (int i = lane; i < half; i += 32) {
        const float2 cs = tb[i];
        const int ia = a.mode == 0 ? i : 2 * i, ib = a.mode == 0 ? i + half : 2 * i + 1;
        const float l = hv[ia], r = hv[ib];
        hv[ia] = l * cs.x - r * cs.y;
        hv[ib] = l * cs.y + r * cs.x;
      }
      __syncwarp();
    }
    __syncthreads();
    if (owns_new) {  // the ring slot of the new position, for later steps
      const int slot = start % a.capacity;
      float *kd = const_cast<float *>(a.k) + ((int64_t)kh * a.capacity + slot) * hd;
      float *vd = const_cast<float *>(a.v) + ((int64_t)kh * a.capacity + slot) * hd;
      for (int d = tid; d < hd; d += ATT_THREADS) { kd[d] = kn_s[d]; vd[d] = vn_s[d]; }
    }
  }

  const int g0 = warp, g1 = warp + ATT_WARPS;
  const bool h0 = g0 < G, h1 = g1 < G;
  float m0 = -FLT_MAX, m1 = -FLT_MAX, l0 = 0.f, l1 = 0.f;
  float4 acc0[NI], acc1[NI];
#pragma unroll
  for (int i = 0; i < NI; i++) acc0[i] = acc1[i] = make_float4(0.f, 0.f, 0.f, 0.f);

  for (int ti = 0; ti < ntiles; ti++) {
    const int tile = p0 + ti * ATT_TILE, cnt = min(ATT_TILE, p1 - tile);
    const int st = nst == 2 ? (ti & 1) : 0;
    if (nst == 2 && ti + 1 < ntiles) cp_async_wait<1>(); else cp_async_wait<0>();
    __syncthreads();
    float *ks = kv_s + (size_t)st * 2 * ATT_TILE * RS, *vs = ks + ATT_TILE * RS;
    if (owns_new && tile + cnt == end) {  // block-uniform
      const int r = end - 1 - tile;
      for (int d = tid; d < hd; d += ATT_THREADS) { ks[r * RS + d] = kn_s[d]; vs[r * RS + d] = vn_s[d]; }
      __syncthreads();
    }
    // scores: lane j <-> key tile + j
    const bool live = lane < cnt;
    float s0 = 0.f, s1 = 0.f;
    {
      const float4 *kr = reinterpret_cast<const float4 *>(ks + lane * RS);
      const float4 *q0 = reinterpret_cast<const float4 *>(q_s + g0 * hd);
      const float4 *q1 = reinterpret_cast<const float4 *>(q_s + (h1 ? g1 : g0) * hd);
#pragma unroll 8
      for (int d4 = 0; d4 < hd4; d4++) {
        const float4 k4 = kr[d4];
        if (h0) {
          const float4 q = q0[d4];
          s0 = fmaf(q.x, k4.x, fmaf(q.y, k4.y, fmaf(q.z, k4.z, fmaf(q.w, k4.w, s0))));
        }
        if (h1) {
          const float4 q = q1[d4];
          s1 = fmaf(q.x, k4.x, fmaf(q.y, k4.y, fmaf(q.z, k4.z, fmaf(q.w, k4.w, s1))));
        }
      }
    }
    float e0 = 0.f, e1 = 0.f;
    if (h0) {
      s0 = live ? s0 * a.scale : -FLT_MAX;
      const float mn = fmaxf(m0, warp_max(s0)), corr = expf(m0 - mn);
      e0 = live ? expf(s0 - mn) : 0.f;
      l0 = fmaf(l0, corr, warp_sum(e0));
      m0 = mn;
#pragma unroll
      for (int i = 0; i < NI; i++) acc0[i] = make_float4(acc0[i].x * corr, acc0[i].y * corr, acc0[i].z * corr, acc0[i].w * corr);
    }
    if (h1) {
      s1 = live ? s1 * a.scale : -FLT_MAX;
      const float mn = fmaxf(m1, warp_max(s1)), corr = expf(m1 - mn);
      e1 = live ? expf(s1 - mn) : 0.f;
      l1 = fmaf(l1, corr, warp_sum(e1));
      m1 = mn;
#pragma unroll
      for (int i = 0; i < NI; i++) acc1[i] = make_float4(acc1[i].x * corr, acc1[i].y * corr, acc1[i].z * corr, acc1[i].w * corr);
    }
    if (h0) {
#pragma unroll 4
      for (int j = 0; j < cnt; j++) {
        const float w0 = __shfl_sync(0xffffffffu, e0, j), w1 = __shfl_sync(0xffffffffu, e1, j);
        const float4 *vr = reinterpret_cast<const float4 *>(vs + j * RS);
#pragma unroll
        for (int i = 0; i < NI; i++) {
          const int d4 = lane + 32 * i;
          if (d4 < hd4) {
            const float4 v = vr[d4];
            acc0[i] = f4_fma(w0, v, acc0[i]);
            if (h1) acc1[i] = f4_fma(w1, v, acc1[i]);
          }
        }
      }
    }
    __syncthreads();  // stage st is free again
    if (nst == 2 && ti + 2 < ntiles) stage(tile + 2 * ATT_TILE, st);
    else if (nst == 1 && ti + 1 < ntiles) stage(tile + ATT_TILE, 0);
  }

  const int pair = t * a.kv_heads + kh;
  float *out_base = a.out + ((int64_t)t * a.heads + kh * G) * hd;
  if (nsp == 1) {
#pragma unroll
    for (int i = 0; i < NI; i++) {
      const int d4 = lane + 32 * i;
      if (d4 < hd4) {
        if (h0) reinterpret_cast<float4 *>(out_base + g0 * hd)[d4] =
            make_float4(acc0[i].x / l0, acc0[i].y / l0, acc0[i].z / l0, acc0[i].w / l0);
        if (h1) reinterpret_cast<float4 *>(out_base + g1 * hd)[d4] =
            make_float4(acc1[i].x / l1, acc1[i].y / l1, acc1[i].z / l1, acc1[i].w / l1);
      }
    }
    pdl_launch_dependents();
    return;
  }
  // partial row per (pair, split, head): acc[hd] | m | l | pad (stride hd + 4)
  const int PR = hd + 4;
  float *part = a.part + ((int64_t)pair * a.splits + sp) * G * PR;
#pragma unroll
  for (int i = 0; i < NI; i++) {
    const int d4 = lane + 32 * i;
    if (d4 < hd4) {
      if (h0) reinterpret_cast<float4 *>(part + g0 * PR)[d4] = acc0[i];
      if (h1) reinterpret_cast<float4 *>(part + g1 * PR)[d4] = acc1[i];
    }
  }
  if (lane == 0) {
    if (h0) { part[g0 * PR + hd] = m0; part[g0 * PR + hd + 1] = l0; }
    if (h1) { part[g1 * PR + hd] = m1; part[g1 * PR + hd + 1] = l1; }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) last_s = atomicAdd(a.ctr + pair, 1u) == (unsigned)(nsp - 1);
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  const float *pb = a.part + (int64_t)pair * a.splits * G * PR;
  const int64_t sstride = (int64_t)G * PR;  // one split
  for (int g = warp; g < G; g += ATT_WARPS) {
    const float *ph = pb + g * PR;
    // split j's weight exp(m_j - M) / sum, held by lane j % 32 (j < 64)
    const float ma = lane < nsp ? __ldcg(ph + lane * sstride + hd) : -FLT_MAX;
    const float mb = lane + 32 < nsp ? __ldcg(ph + (lane + 32) * sstride + hd) : -FLT_MAX;
    const float M = warp_max(fmaxf(ma, mb));
    const float wa = lane < nsp ? expf(ma - M) : 0.f, wb = lane + 32 < nsp ? expf(mb - M) : 0.f;
    const float la = lane < nsp ? __ldcg(ph + lane * sstride + hd + 1) : 0.f;
    const float lb = lane + 32 < nsp ? __ldcg(ph + (lane + 32) * sstride + hd + 1) : 0.f;
    const float den = warp_sum(fmaf(wa, la, wb * lb));
#pragma unroll
    for (int i = 0; i < NI; i++) {
      const int d4 = lane + 32 * i;
      float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
      for (int j = 0; j < nsp; j++) {
        const float w = __shfl_sync(0xffffffffu, j < 32 ? wa : wb, j & 31);
        if (d4 < hd4) num = f4_fma(w, __ldcg(reinterpret_cast<const float4 *>(ph + j * sstride) + d4), num);
      }
      if (d4 < hd4) reinterpret_cast<float4 *>(out_base + g * hd)[d4] = make_float4(num.x / den, num.y / den, num.z / den, num.w / den);
    }
  }
  if (tid == 0) a.ctr[pair] = 0u;
  pdl_launch_dependents();
}

// Prompt-batch attention (n > 1 rows, no fused RoPE): one CTA per (block of
// ATR_ROWS consecutive query rows, kv head, key split) stages each K/V tile
// once for all ATR_ROWS * G query heads of the block (the decode kernel above
// would read every tile once per row). Warp w owns query-head vectors
// qh = w + 8i (qh = row * G + head); lane j scores key j of the tile with the
// row's causal window as mask; the online softmax and the PV accumulation are
// the decode kernel's, per vector. Splits of at least ATR_MIN_CHUNK keys are
// merged by the CTA of the block that arrives last (same partial layout).
constexpr int ATR_ROWS = 8, ATR_THREADS = 256, ATR_WARPS = 8, ATR_MIN_CHUNK = 128;

// GM: the largest group size (query heads per kv head) the instance handles (4 or 8),
// so that the per-vector registers of the smaller groups leave room for two CTAs per SM.
template <int NI, int GM>
__global__ void __launch_bounds__(ATR_THREADS, GM <= 4 ? 2 : 1) attention_rows_kernel(const AttnArgs a) {
  extern __shared__ __align__(16) float sm[];
  const int G = a.heads / a.kv_heads, hd = a.hd, hd4 = hd >> 2, RS = hd + 4;
  const int QH = ATR_ROWS * G;
  float *q_s = sm;             // [QH][hd]
  float *kv_s = q_s + QH * hd; // [2][K|V][ATT_TILE][RS]
  __shared__ int last_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int qb = blockIdx.x / a.kv_heads, kh = blockIdx.x % a.kv_heads, sp = blockIdx.y;
  pdl_wait();
  const int start = a.start ? *a.start : a.start_host;
  const int t0 = qb * ATR_ROWS, nrows = min(ATR_ROWS, a.n - t0);
  // the block's key range: from the first row's window start to the last row's position
  const int end_first = start + t0 + 1, kmin = end_first - (end_first < a.window ? end_first : a.window);
  const int kmax = start + t0 + nrows, L = kmax - kmin;
  int chunk = (L + (int)gridDim.y - 1) / (int)gridDim.y;  // gridDim.y <= a.splits (the partial stride)
  if (chunk < ATR_MIN_CHUNK) chunk = ATR_MIN_CHUNK;
  const int nsp = (L + chunk - 1) / chunk;
  if (sp >= nsp) return;
  const int p0 = kmin + sp * chunk, p1 = min(kmax, p0 + chunk);
  const float *kb = a.k + (int64_t)kh * a.capacity * hd;
  const float *vb = a.v + (int64_t)kh * a.capacity * hd;
  const int ntiles = (p1 - p0 + ATT_TILE - 1) / ATT_TILE;

  auto stage = [&](int tile, int st) {
    const int cnt = min(ATT_TILE, p1 - tile), total = cnt * hd4;
    float *ks = kv_s + (size_t)st * 2 * ATT_TILE * RS, *vs = ks + ATT_TILE * RS;
    for (int i = tid; i < total; i += ATR_THREADS) {
      const int r = i / hd4, c = (i - r * hd4) * 4;
      const int64_t row = (int64_t)((tile + r) % a.capacity) * hd;
      cp_async16(ks + r * RS + c, kb + row + c);
      cp_async16(vs + r * RS + c, vb + row + c);
    }
    cp_async_commit();
  };
  stage(p0, 0);
  if (ntiles > 1) stage(p0 + ATT_TILE, 1);
  for (int i = tid; i < QH * hd4; i += ATR_THREADS) {
    const int qh = i / hd4, d4 = i - qh * hd4, r = qh / G, g = qh - r * G;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < nrows) v = reinterpret_cast<const float4 *>(a.q + ((int64_t)(t0 + r) * a.heads + kh * G + g) * hd)[d4];
    reinterpret_cast<float4 *>(q_s + qh * hd)[d4] = v;
  }

  // this warp's vectors: qh = warp + 8i, i < G (row r = qh / G); row r's keys are
  // [P_r + 1 - min(P_r + 1, window), P_r] with P_r = start + t0 + r
  float m[GM], l[GM];
  float4 acc[GM][NI];
  int lo[GM], hi[GM];
#pragma unroll
  for (int i = 0; i < GM; i++) {
    m[i] = -FLT_MAX;
    l[i] = 0.f;
#pragma unroll
    for (int k = 0; k < NI; k++) acc[i][k] = make_float4(0.f, 0.f, 0.f, 0.f);
    const int qh = warp + ATR_WARPS * i, r = qh / G;
    const int P = start + t0 + r, e = P + 1;
    hi[i] = r < nrows ? P : -1;  // dead vectors (past the last row) match no key
    lo[i] = e - (e < a.window ? e : a.window);
  }

  for (int ti = 0; ti < ntiles; ti++) {
    const int tile = p0 + ti * ATT_TILE, cnt = min(ATT_TILE, p1 - tile), st = ti & 1;
    if (ti + 1 < ntiles) cp_async_wait<1>(); else cp_async_wait<0>();
    __syncthreads();
    const float *ks = kv_s + (size_t)st * 2 * ATT_TILE * RS, *vs = ks + ATT_TILE * RS;
    const int key = tile + lane;
    float sc[GM];
#pragma unroll
    for (int i = 0; i < GM; i++) sc[i] = 0.f;
    {
      const float4 *kr = reinterpret_cast<const float4 *>(ks + lane * RS);
#pragma unroll 4
      for (int d4 = 0; d4 < hd4; d4++) {
        const float4 k4 = kr[d4];
#pragma unroll
        for (int i = 0; i < GM; i++) {
          if (i < G) {
            const float4 q = reinterpret_cast<const float4 *>(q_s + (warp + ATR_WARPS * i) * hd)[d4];
            sc[i] = fmaf(q.x, k4.x, fmaf(q.y, k4.y, fmaf(q.z, k4.z, fmaf(q.w, k4.w, sc[i]))));
          }
        }
      }
    }
    float e[GM];
#pragma unroll
    for (int i = 0; i < GM; i++) {
      e[i] = 0.f;
      if (i < G) {
        const bool live = lane < cnt && key >= lo[i] && key <= hi[i];
        const float s_ = live ? sc[i] * a.scale : -FLT_MAX;
        const float mn = fmaxf(m[i], warp_max(s_)), corr = expf(m[i] - mn);
        e[i] = live ? expf(s_ - mn) : 0.f;
        l[i] = fmaf(l[i], corr, warp_sum(e[i]));
        m[i] = mn;
#pragma unroll
        for (int k = 0; k < NI; k++) acc[i][k] = make_float4(acc[i][k].x * corr, acc[i][k].y * corr, acc[i][k].z * corr, acc[i][k].w * corr);
      }
    }
#pragma unroll 2
    for (int j = 0; j < cnt; j++) {
      const float4 *vr = reinterpret_cast<const float4 *>(vs + j * RS);
      float4 v[NI];
#pragma unroll
      for (int k = 0; k < NI; k++) {
        const int d4 = lane + 32 * k;
        v[k] = d4 < hd4 ? vr[d4] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int i = 0; i < GM; i++) {
        if (i < G) {
          const float w = __shfl_sync(0xffffffffu, e[i], j);
#pragma unroll
          for (int k = 0; k < NI; k++) acc[i][k] = f4_fma(w, v[k], acc[i][k]);
        }
      }
    }
    __syncthreads();  // stage st is free again
    if (ti + 2 < ntiles) stage(tile + 2 * ATT_TILE, st);
  }

  const int PR = hd + 4;
  if (nsp == 1) {
#pragma unroll
    for (int i = 0; i < GM; i++) {
      const int qh = warp + ATR_WARPS * i, r = qh / G, g = qh - r * G;
      if (i >= G || r >= nrows) continue;
      float *o = a.out + ((int64_t)(t0 + r) * a.heads + kh * G + g) * hd;
#pragma unroll
      for (int k = 0; k < NI; k++) {
        const int d4 = lane + 32 * k;
        if (d4 < hd4)
          reinterpret_cast<float4 *>(o)[d4] = make_float4(acc[i][k].x / l[i], acc[i][k].y / l[i], acc[i][k].z / l[i], acc[i][k].w / l[i]);
      }
    }
    pdl_launch_dependents();
    return;
  }
  // partial rows: [(row * kv_heads + kh) * splits + sp][g] of acc | m | l | pad
#pragma unroll
  for (int i = 0; i < GM; i++) {
    const int qh = warp + ATR_WARPS * i, r = qh / G, g = qh - r * G;
    if (i >= G || r >= nrows) continue;
    float *part = a.part + (((int64_t)(t0 + r) * a.kv_heads + kh) * a.splits + sp) * G * PR + g * PR;
#pragma unroll
    for (int k = 0; k < NI; k++) {
      const int d4 = lane + 32 * k;
      if (d4 < hd4) reinterpret_cast<float4 *>(part)[d4] = acc[i][k];
    }
    if (lane == 0) {
      part[hd] = m[i];
      part[hd + 1] = l[i];
    }
  }
  __threadfence();
  __syncthreads();
  const int pair = qb * a.kv_heads + kh;
  if (tid == 0) last_s = atomicAdd(a.ctr + pair, 1u) == (unsigned)(nsp - 1);
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  const int64_t sstride = (int64_t)G * PR;
  for (int qh = warp; qh < nrows * G; qh += ATR_WARPS) {
    const int r = qh / G, g = qh - r * G;
    const float *ph = a.part + ((int64_t)(t0 + r) * a.kv_heads + kh) * a.splits * sstride + g * PR;
    const float ma = lane < nsp ? __ldcg(ph + lane * sstride + hd) : -FLT_MAX;
    const float mb = lane + 32 < nsp ? __ldcg(ph + (lane + 32) * sstride + hd) : -FLT_MAX;
    const float M = warp_max(fmaxf(ma, mb));
    const float wa = lane < nsp ? expf(ma - M) : 0.f, wb = lane + 32 < nsp ? expf(mb - M) : 0.f;
    const float la = lane < nsp ? __ldcg(ph + lane * sstride + hd + 1) : 0.f;
    const float lb = lane + 32 < nsp ? __ldcg(ph + (lane + 32) * sstride + hd + 1) : 0.f;
    const float den = warp_sum(fmaf(wa, la, wb * lb));
    float *o = a.out + ((int64_t)(t0 + r) * a.heads + kh * G + g) * hd;
#pragma unroll
    for (int k = 0; k < NI; k++) {
      const int d4 = lane + 32 * k;
      float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int j = 0; j < nsp; j++) {
        const float w = __shfl_sync(0xffffffffu, j < 32 ? wa : wb, j & 31);
        if (d4 < hd4) num = f4_fma(w, __ldcg(reinterpret_cast<const float4 *>(ph + j * sstride) + d4), num);
      }
      if (d4 < hd4) reinterpret_cast<float4 *>(o)[d4] = make_float4(num.x / den, num.y / den, num.z / den, num.w / den);
    }
  }
  if (tid == 0) a.ctr[pair] = 0u;
  pdl_launch_dependents();
}

template <int NI, int GM>
static cudaError_t launch_attention_rows_ni(const AttnArgs &a, size_t smem, cudaStream_t s, bool pdl) {
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(attention_rows_kernel<NI, GM>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const int blocks = (a.n + ATR_ROWS - 1) / ATR_ROWS;
  // no block reads more than capacity keys: splits beyond that many chunks would exit at once
  const int ysplits = min(a.splits, (a.capacity + ATR_MIN_CHUNK - 1) / ATR_MIN_CHUNK);
  return launch_k(attention_rows_kernel<NI, GM>, dim3(blocks * a.kv_heads, ysplits), dim3(ATR_THREADS), smem, s, pdl, a);
}

template <int NI>
static cudaError_t launch_attention_ni(const AttnArgs &a, size_t smem, cudaStream_t s, bool pdl) {
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(attention_kernel<NI>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  return launch_k(attention_kernel<NI>, dim3(a.n * a.kv_heads, a.splits), dim3(ATT_THREADS), smem, s, pdl, a);
}

cudaError_t launch_attention(const AttnArgs &a, cudaStream_t s, bool pdl) {
  const int G = a.heads / a.kv_heads;
  if (G > ATT_GMAX || a.hd % 4 || a.hd > 4 * ATT_THREADS || a.splits < 1 || a.splits > ATT_MAXSPLIT) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(a.k) | reinterpret_cast<uintptr_t>(a.v) | reinterpret_cast<uintptr_t>(a.out) |
       reinterpret_cast<uintptr_t>(a.part)) & 15)
    return cudaErrorMisalignedAddress;
  if (a.n > 1 && !a.qkv && a.hd <= 256) {  // prompt batch: K/V tiles shared by ATR_ROWS query rows
    const size_t smem = sizeof(float) * ((size_t)ATR_ROWS * G * a.hd + 2 * 2 * ATT_TILE * (size_t)(a.hd + 4));
    if (a.hd <= 128) return G <= 4 ? launch_attention_rows_ni<1, 4>(a, smem, s, pdl) : launch_attention_rows_ni<1, 8>(a, smem, s, pdl);
    return G <= 4 ? launch_attention_rows_ni<2, 4>(a, smem, s, pdl) : launch_attention_rows_ni<2, 8>(a, smem, s, pdl);
  }
  const int nst = a.hd <= 256 ? 2 : 1;
  const size_t smem = sizeof(float) * ((size_t)G * a.hd + 2 * (size_t)a.hd + (size_t)nst * 2 * ATT_TILE * (a.hd + 4));
  if (a.hd <= 128) return launch_attention_ni<1>(a, smem, s, pdl);
  if (a.hd <= 256) return launch_attention_ni<2>(a, smem, s, pdl);
  return launch_attention_ni<4>(a, smem, s, pdl);
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
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) y[i] = __ldcg(y + i) + x[i];
  pdl_launch_dependents();
}
cudaError_t launch_add(const float *x, float *y, int64_t n, cudaStream_t s, bool pdl) {
  if (n <= 0) return cudaSuccess;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  return launch_k(add_kernel, dim3((unsigned)blocks), dim3(256), 0, s, pdl, x, y, n);
}

}  // namespace wgd
