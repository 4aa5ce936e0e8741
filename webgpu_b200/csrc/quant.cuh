// Block codecs for the device row layouts (see common.cuh: dev_row_bytes).
//
// Two views of every GGML type the reference decodes (quant.ts:6-29 and the
// WGSL weightFunction, shaders.ts:13-38 of the reference project):
//
//  * dequant_elem<T>: one value, bit-exact with the WGSL f32 expression order
//    (each product and difference rounded separately, no FMA contraction).
//
//  * Codec<T>::dot: the GEMV inner product over one 32-value "unit" that one
//    lane owns. A unit is two runs of 16 columns (colA.., colB..); the lane
//    keeps those 32 activations in registers for every row it visits. The
//    weight integers q are turned into the exact affine image f = 0.5 + q/256
//    with a single PRMT (q < 128 placed in byte 2 under exponent 0x3F), so
//       sum_i q_i x_i = 256 * sum_i f_i x_i - 128 * sum_i x_i
//    with only fp32 rounding; per-block scales are applied once per run:
//       sum_i (d*sc*q_i - dmin*mn) x_i = d*sc*sum(q x) - dmin*mn*sum(x).
//    This is an algebraic regrouping of the reference sum; results agree
//    with the f64 oracle within fp32 tolerance, not bit for bit.
#pragma once
#include "common.cuh"

namespace wgd {

template <int T>
__host__ __device__ constexpr int block_elems_dev() { return T == F32 || T == F16 ? 1 : (T == Q4_0 || T == Q8_0) ? 32 : 256; }

// ----------------------------------------------------------- bit-exact dequant

template <int T>
__device__ __forceinline__ float dequant_elem(const uint8_t *row, int nb, int col);

template <> __device__ __forceinline__ float dequant_elem<F32>(const uint8_t *row, int, int col) {
  return __ldg(reinterpret_cast<const float *>(row) + col);
}
template <> __device__ __forceinline__ float dequant_elem<F16>(const uint8_t *row, int, int col) {
  return h2f(__ldg(reinterpret_cast<const unsigned short *>(row) + col));
}
template <> __device__ __forceinline__ float dequant_elem<Q4_0>(const uint8_t *row, int nb, int col) {
  int b = col >> 5, j = col & 31;
  float d = h2f(__ldg(reinterpret_cast<const unsigned short *>(row + 16 * nb) + b));
  uint32_t q = (__ldg(row + 16 * b + (j & 15)) >> ((j >> 4) * 4)) & 15u;
  return __fmul_rn(d, (float)((int)q - 8));
}
template <> __device__ __forceinline__ float dequant_elem<Q8_0>(const uint8_t *row, int nb, int col) {
  int b = col >> 5, j = col & 31;
  float d = h2f(__ldg(reinterpret_cast<const unsigned short *>(row + 32 * nb) + b));
  return __fmul_rn(d, (float)(int8_t)__ldg(row + 32 * b + j));
}
__device__ __forceinline__ void k_scale_min(const uint8_t *S, int s, uint32_t &sc, uint32_t &mn) {
  if (s < 4) { sc = __ldg(S + s) & 63u; mn = __ldg(S + 4 + s) & 63u; }
  else {
    sc = (__ldg(S + 4 + s) & 15u) | ((__ldg(S + s - 4) >> 6u) << 4u);
    mn = (__ldg(S + 4 + s) >> 4u) | ((__ldg(S + s) >> 6u) << 4u);
  }
}
template <int T>
__device__ __forceinline__ float dequant_k(const uint8_t *row, int col) {
  constexpr int BB = T == Q4_K ? 144 : 176;
  int sb = col >> 8, j = col & 255, s = j >> 5;
  const uint8_t *p = row + (int64_t)sb * BB;
  float d = h2f(__ldg(reinterpret_cast<const unsigned short *>(p)));
  float dmin = h2f(__ldg(reinterpret_cast<const unsigned short *>(p) + 1));
  uint32_t sc, mn;
  k_scale_min(p + 4, s, sc, mn);
  uint32_t q = (__ldg(p + (T == Q4_K ? 16 : 48) + (j >> 6) * 32 + (j & 31)) >> ((s & 1) * 4)) & 15u;
  if (T == Q5_K) q |= ((__ldg(p + 16 + (j & 31)) >> s) & 1u) << 4;
  return __fsub_rn(__fmul_rn(d, (float)(sc * q)), __fmul_rn(dmin, (float)mn));
}
template <> __device__ __forceinline__ float dequant_elem<Q4_K>(const uint8_t *row, int, int col) { return dequant_k<Q4_K>(row, col); }
template <> __device__ __forceinline__ float dequant_elem<Q5_K>(const uint8_t *row, int, int col) { return dequant_k<Q5_K>(row, col); }
template <> __device__ __forceinline__ float dequant_elem<Q6_K>(const uint8_t *row, int nb, int col) {
  int sb = col >> 8, j = col & 255;
  int segment = j >> 7, quarter = (j & 127) >> 5, lane = j & 31;
  const uint8_t *p = row + (int64_t)sb * 208;
  uint32_t low = (__ldg(p + segment * 64 + (quarter & 1) * 32 + lane) >> ((quarter >> 1) * 4)) & 15u;
  uint32_t high = (__ldg(p + 128 + segment * 32 + lane) >> (quarter * 2)) & 3u;
  int sc = (int8_t)__ldg(p + 192 + segment * 8 + quarter * 2 + (lane >> 4));
  float d = h2f(__ldg(reinterpret_cast<const unsigned short *>(row + 208 * nb) + sb));
  return __fmul_rn(__fmul_rn(d, (float)sc), (float)((int)(low | (high << 4)) - 32));
}

// ------------------------------------------------------------ GEMV unit codecs

__device__ __forceinline__ uint32_t pick4(const uint4 &v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// One decoded unit: 32 weight images f (run A = f[0..15], run B = f[16..31]) and
// the coefficients that turn run dot products into the unit's contribution:
//   contribution = qa * sum(fA x) + xa * sum(xA) + qb * sum(fB x) + xb * sum(xB).
struct Unit {
  float f[32];
  float qa, xa, qb, xb;
};

// The activations one lane owns for one unit, and their run sums.
struct XUnit {
  float a[16], b[16];
  float sa, sb;
};

__device__ __forceinline__ float unit_apply(const Unit &w, const XUnit &x) {
  float2 pa = make_float2(0.f, 0.f), pb = make_float2(0.f, 0.f), pc = make_float2(0.f, 0.f), pd = make_float2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < 16; i += 4) {
    pa = __ffma2_rn(make_float2(w.f[i], w.f[i + 1]), make_float2(x.a[i], x.a[i + 1]), pa);
    pc = __ffma2_rn(make_float2(w.f[i + 2], w.f[i + 3]), make_float2(x.a[i + 2], x.a[i + 3]), pc);
    pb = __ffma2_rn(make_float2(w.f[16 + i], w.f[17 + i]), make_float2(x.b[i], x.b[i + 1]), pb);
    pd = __ffma2_rn(make_float2(w.f[18 + i], w.f[19 + i]), make_float2(x.b[i + 2], x.b[i + 3]), pd);
  }
  float sa = (pa.x + pa.y) + (pc.x + pc.y), sb = (pb.x + pb.y) + (pd.x + pd.y);
  return fmaf(w.qa, sa, fmaf(w.xa, x.sa, fmaf(w.qb, sb, w.xb * x.sb)));
}

// Four bytes (each < 128) -> four affine images 0.5 + b/256.
__device__ __forceinline__ void affine4(uint32_t word, float *f) {
  f[0] = byte_as_affine(word, sel_byte(0));
  f[1] = byte_as_affine(word, sel_byte(1));
  f[2] = byte_as_affine(word, sel_byte(2));
  f[3] = byte_as_affine(word, sel_byte(3));
}

template <int T> struct Codec;

// F32: unit u = columns 32u .. 32u+31 (runs 32u and 32u+16).
template <> struct Codec<F32> {
  static __device__ __forceinline__ void cols(int u, int &ca, int &cb) { ca = 32 * u; cb = ca + 16; }
  static __device__ __forceinline__ void decode(const uint8_t *row, int, int u, Unit &o) {
    const uint8_t *p = row + 128 * u;
#pragma unroll
    for (int k = 0; k < 8; k++) {
      uint4 v = ldg_stream(p + 16 * k);
      o.f[4 * k] = __uint_as_float(v.x); o.f[4 * k + 1] = __uint_as_float(v.y);
      o.f[4 * k + 2] = __uint_as_float(v.z); o.f[4 * k + 3] = __uint_as_float(v.w);
    }
    o.qa = 1.f; o.xa = 0.f; o.qb = 1.f; o.xb = 0.f;
  }
};

template <> struct Codec<F16> {
  static __device__ __forceinline__ void cols(int u, int &ca, int &cb) { ca = 32 * u; cb = ca + 16; }
  static __device__ __forceinline__ void decode(const uint8_t *row, int, int u, Unit &o) {
    const uint8_t *p = row + 64 * u;
#pragma unroll
    for (int k = 0; k < 4; k++) {
      uint4 v = ldg_stream(p + 16 * k);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int m = 0; m < 4; m++) {
        float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[m]));
        o.f[8 * k + 2 * m] = f.x; o.f[8 * k + 2 * m + 1] = f.y;
      }
    }
    o.qa = 1.f; o.xa = 0.f; o.qb = 1.f; o.xb = 0.f;
  }
};

// Q4_0: unit = one 32-value block; byte i holds value i (low nibble) and i+16 (high).
template <> struct Codec<Q4_0> {
  static __device__ __forceinline__ void cols(int u, int &ca, int &cb) { ca = 32 * u; cb = ca + 16; }
  static __device__ __forceinline__ void decode(const uint8_t *row, int nb, int u, Unit &o) {
    uint4 q = ldg_stream(row + 16 * u);
    float d = h2f(ldg_u16(row + 16 * nb + 2 * u));
    const uint32_t m = 0x0F0F0F0Fu, w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int k = 0; k < 4; k++) { affine4(w[k] & m, o.f + 4 * k); affine4((w[k] >> 4) & m, o.f + 16 + 4 * k); }
    // sum (q-8) x = 256 f - (128 + 8) sum x
    o.qa = 256.f * d; o.xa = -136.f * d; o.qb = o.qa; o.xb = o.xa;
  }
};

// Q8_0: unit = one block of 32 signed bytes; values are converted exactly
// (byte^0x80 placed under exponent 0x4B40 gives 1.5*2^23 + b + 128).
template <> struct Codec<Q8_0> {
  static __device__ __forceinline__ void cols(int u, int &ca, int &cb) { ca = 32 * u; cb = ca + 16; }
  static __device__ __forceinline__ void decode(const uint8_t *row, int nb, int u, Unit &o) {
    uint4 q0 = ldg_stream(row + 32 * u), q1 = ldg_stream(row + 32 * u + 16);
    float d = h2f(ldg_u16(row + 32 * nb + 2 * u));
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    const float2 off = make_float2(-12583040.f, -12583040.f);
#pragma unroll
    for (int m = 0; m < 8; m++) {
      uint32_t t = w[m] ^ 0x80808080u;
#pragma unroll
      for (int k = 0; k < 4; k += 2) {
        uint32_t r0, r1;
        asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r0) : "r"(t), "r"(0x4B40u), "r"(0x5460u | (uint32_t)k));
        asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r1) : "r"(t), "r"(0x4B40u), "r"(0x5460u | (uint32_t)(k + 1)));
        float2 v = __fadd2_rn(make_float2(__uint_as_float(r0), __uint_as_float(r1)), off);
        o.f[4 * m + k] = v.x; o.f[4 * m + k + 1] = v.y;
      }
    }
    o.qa = d; o.xa = 0.f; o.qb = d; o.xb = 0.f;
  }
};

// Q4_K / Q5_K: unit u -> super-block u/8, 16-byte quant chunk c = u%8; the chunk's
// low nibbles are sub-block 2g (columns 64g+16h..), high nibbles sub-block 2g+1
// (columns 64g+32+16h..), g = c/2, h = c%2.
__device__ __forceinline__ void k_scales2(const uint4 &hdr, int g, float &sc0, float &mn0, float &sc1, float &mn1) {
  // S bytes: S[0..3] = hdr.y, S[4..7] = hdr.z, S[8..11] = hdr.w. Sub-blocks s0 = 2g, s1 = 2g+1.
  int k0 = (2 * g) & 3;
  uint32_t A = hdr.y >> (8 * k0), B = hdr.z >> (8 * k0), C = hdr.w >> (8 * k0);
  uint32_t a0 = A & 255u, a1 = (A >> 8) & 255u, b0 = B & 255u, b1 = (B >> 8) & 255u, c0 = C & 255u, c1 = (C >> 8) & 255u;
  bool hi = g >= 2;
  uint32_t s0 = hi ? ((c0 & 15u) | ((a0 >> 6) << 4)) : (a0 & 63u);
  uint32_t m0 = hi ? ((c0 >> 4) | ((b0 >> 6) << 4)) : (b0 & 63u);
  uint32_t s1 = hi ? ((c1 & 15u) | ((a1 >> 6) << 4)) : (a1 & 63u);
  uint32_t m1 = hi ? ((c1 >> 4) | ((b1 >> 6) << 4)) : (b1 & 63u);
  sc0 = (float)s0; mn0 = (float)m0; sc1 = (float)s1; mn1 = (float)m1;
}

template <> struct Codec<Q4_K> {
  static __device__ __forceinline__ void cols(int u, int &ca, int &cb) {
    int sb = u >> 3, c = u & 7, g = c >> 1, h = c & 1;
    ca = 256 * sb + 64 * g + 16 * h; cb = ca + 32;
  }
  static __device__ __forceinline__ void decode(const uint8_t *row, int, int u, Unit &o) {
    int sb = u >> 3, c = u & 7;
    const uint8_t *blk = row + 144 * sb;
    uint4 q = ldg_stream(blk + 16 + 16 * c);
    uint4 hdr = ldg_cached(blk);
    float d = h2f(hdr.x), dm = h2f(hdr.x >> 16);
    float sc0, mn0, sc1, mn1;
    k_scales2(hdr, c >> 1, sc0, mn0, sc1, mn1);
    const uint32_t m = 0x0F0F0F0Fu, w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int k = 0; k < 4; k++) { affine4(w[k] & m, o.f + 4 * k); affine4((w[k] >> 4) & m, o.f + 16 + 4 * k); }
    // d*sc*(256 f - 128 sum x) - dmin*mn*sum x
    float da = d * sc0, db = d * sc1;
    o.qa = 256.f * da; o.xa = -fmaf(128.f, da, dm * mn0);
    o.qb = 256.f * db; o.xb = -fmaf(128.f, db, dm * mn1);
  }
};

template <> struct Codec<Q5_K> {
  static __device__ __forceinline__ void cols(int u, int &ca, int &cb) { Codec<Q4_K>::cols(u, ca, cb); }
  static __device__ __forceinline__ void decode(const uint8_t *row, int, int u, Unit &o) {
    int sb = u >> 3, c = u & 7, g = c >> 1, h = c & 1;
    const uint8_t *blk = row + 176 * sb;
    uint4 q = ldg_stream(blk + 48 + 16 * c);
    uint4 qh = ldg_cached(blk + 16 + 16 * h);
    uint4 hdr = ldg_cached(blk);
    float d = h2f(hdr.x), dm = h2f(hdr.x >> 16);
    float sc0, mn0, sc1, mn1;
    k_scales2(hdr, g, sc0, mn0, sc1, mn1);
    const uint32_t m = 0x0F0F0F0Fu, one = 0x01010101u;
    const uint32_t w[4] = {q.x, q.y, q.z, q.w}, hw[4] = {qh.x, qh.y, qh.z, qh.w};
    const int s0 = 2 * g, s1 = 2 * g + 1;
#pragma unroll
    for (int k = 0; k < 4; k++) {
      affine4((w[k] & m) | (((hw[k] >> s0) & one) << 4), o.f + 4 * k);
      affine4(((w[k] >> 4) & m) | (((hw[k] >> s1) & one) << 4), o.f + 16 + 4 * k);
    }
    float da = d * sc0, db = d * sc1;
    o.qa = 256.f * da; o.xa = -fmaf(128.f, da, dm * mn0);
    o.qb = 256.f * db; o.xb = -fmaf(128.f, db, dm * mn1);
  }
};

// Q6_K: unit u -> super-block u/8, ql chunk c = u%8: segment = c/4, quarter pair
// qp = (c/2)%2, half h = c%2. Low nibbles are quarter qp, high nibbles quarter qp+2.
template <> struct Codec<Q6_K> {
  static __device__ __forceinline__ void cols(int u, int &ca, int &cb) {
    int sb = u >> 3, c = u & 7, seg = c >> 2, qp = (c >> 1) & 1, h = c & 1;
    ca = 256 * sb + 128 * seg + 32 * qp + 16 * h; cb = ca + 64;
  }
  static __device__ __forceinline__ void decode(const uint8_t *row, int nb, int u, Unit &o) {
    int sb = u >> 3, c = u & 7, seg = c >> 2, qp = (c >> 1) & 1, h = c & 1;
    const uint8_t *blk = row + 208 * sb;
    uint4 ql = ldg_stream(blk + 64 * seg + 32 * qp + 16 * h);
    uint4 qh = ldg_cached(blk + 128 + 32 * seg + 16 * h);
    uint4 scv = ldg_cached(blk + 192);
    float d = h2f(ldg_u16(row + 208 * nb + 2 * sb));
    // scale bytes: index 8*seg + 2*quarter + h, for quarter qp (A) and qp+2 (B = A + 4).
    int ia = 8 * seg + 2 * qp + h;
    uint32_t wa = pick4(scv, ia >> 2), wb = pick4(scv, (ia >> 2) + 1);
    float sca = (float)(int8_t)((wa >> (8 * (ia & 3))) & 255u);
    float scb = (float)(int8_t)((wb >> (8 * (ia & 3))) & 255u);
    const uint32_t m = 0x0F0F0F0Fu, three = 0x03030303u;
    const uint32_t w[4] = {ql.x, ql.y, ql.z, ql.w}, hw[4] = {qh.x, qh.y, qh.z, qh.w};
    const int sa = 2 * qp, sbh = 2 * qp + 4;
#pragma unroll
    for (int k = 0; k < 4; k++) {
      affine4((w[k] & m) | (((hw[k] >> sa) & three) << 4), o.f + 4 * k);
      affine4(((w[k] >> 4) & m) | (((hw[k] >> sbh) & three) << 4), o.f + 16 + 4 * k);
    }
    // sum (q-32) x = 256 f - (128 + 32) sum x
    float da = d * sca, db = d * scb;
    o.qa = 256.f * da; o.xa = -160.f * da; o.qb = 256.f * db; o.xb = -160.f * db;
  }
};

// ----------------------------------------------------------- repack raw -> dev

// Moves one GGUF block (raw, `bb` bytes) into the device row layout. `bi` is the
// block's index within the destination row, `nbl` the destination row's block count.
__device__ __forceinline__ void repack_block(int type, const uint8_t *src, uint8_t *dst_row, int bi, int nbl) {
  switch (type) {
    case F32: for (int i = 0; i < 4; i++) dst_row[4 * bi + i] = src[i]; break;
    case F16: dst_row[2 * bi] = src[0]; dst_row[2 * bi + 1] = src[1]; break;
    case Q4_0:
      for (int i = 0; i < 16; i++) dst_row[16 * bi + i] = src[2 + i];
      dst_row[16 * nbl + 2 * bi] = src[0]; dst_row[16 * nbl + 2 * bi + 1] = src[1];
      break;
    case Q8_0:
      for (int i = 0; i < 32; i++) dst_row[32 * bi + i] = src[2 + i];
      dst_row[32 * nbl + 2 * bi] = src[0]; dst_row[32 * nbl + 2 * bi + 1] = src[1];
      break;
    case Q4_K: for (int i = 0; i < 144; i++) dst_row[144 * bi + i] = src[i]; break;
    case Q5_K: for (int i = 0; i < 176; i++) dst_row[176 * bi + i] = src[i]; break;
    case Q6_K:
      for (int i = 0; i < 208; i++) dst_row[208 * bi + i] = src[i];
      dst_row[208 * nbl + 2 * bi] = src[208]; dst_row[208 * nbl + 2 * bi + 1] = src[209];
      break;
  }
}

}  // namespace wgd
