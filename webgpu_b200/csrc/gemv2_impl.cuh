// Tensor-core dequant GEMV over the tile-16 layout (tile.cuh), for decode.
//
// Exact integer inner products on the tensor cores (mma.sync u8 x s8 -> s32):
// the weight quants q stay integers, and every 256-column block of each fp32
// activation row is written as three int8 digit planes with one scale,
//     x ~= s * (a + b/254 + c/254^2),   s = max|x| / 127 over the block,
// which reproduces x to ~6e-8 of the block maximum. One MMA column holds one
// digit plane, so an m16n8 tile yields sum(q*a), sum(q*b), sum(q*c) for 16
// weight rows and up to two activation rows. Because the digit unit is shared
// by the whole super-block, the integer results of its sub-blocks are combined
// in int32 with the integer sub-block scales before one conversion:
//   Q4_K: sum_j (d*sc_j*q - dmin*mn_j) x = s*(d*sum_j sc_j*D_j - dmin*sum_j mn_j*Sdig_j)
//   Q6_K: sum_j d*sc_j*(q-32) x          = s*d*sum_j sc_j*(D_j - 32*Sdig_j)
// (Sdig_j = digit sum of the activation over sub-block j). All int32 ranges are
// bounded well inside 2^31 (see the comments at each accumulation).
//
// Work split (stream-K at warp granularity): the matrix's (tile, K-chunk)
// units are cut into equal contiguous ranges, one per warp of a persistent
// grid. A warp owns whole 16-row tiles where its range covers them and writes
// them directly; a tile cut between warps is finished by the warp that
// arrives last, which sums the partials in worker order (deterministic).
// Each warp requests its first chunk before the programmatic-launch wait and
// keeps one chunk in flight while it computes the other.
#pragma once
#include "kernels.h"
#include "tile.cuh"

namespace wgd {

constexpr int G2_WARPS = 8;

struct Gemv2Args {
  const uint8_t *w;  // tiled weights
  int rows, cols, tiles, nkb;
  const float *x;
  int ldx;
  const float *norm_w;
  float eps;
  float *y;
  int ldy;
  const float *bias;
  int epi;
  int batch;
  float *part;         // [tiles][maxc][16 * NB] partial row sums of split tiles
  unsigned *tile_ctr;  // [tiles] zeroed arrival counters (left zeroed)
  int maxc;            // partial slots per tile
};

__device__ __forceinline__ void mma_k32(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void mma_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm("mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%8,%9,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(b0), "r"(0), "r"(0), "r"(0), "r"(0));
}
// byte k of a word as an unsigned / sign-extended 32-bit integer
__device__ __forceinline__ int ubyte(uint32_t w, int k) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(w), "r"(0u), "r"(0x4440u | (uint32_t)k));
  return (int)r;
}
__device__ __forceinline__ int sbyte(uint32_t w, int k) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(w), "r"(0u), "r"(0x0000u | (uint32_t)k | ((uint32_t)(k | 8) << 4) |
                                                               ((uint32_t)(k | 8) << 8) | ((uint32_t)(k | 8) << 12)));
  return (int)r;
}

__device__ __forceinline__ float g2_silu(float g) { return g / (1.0f + expf(-g)); }
__device__ __forceinline__ float g2_gelu(float x) {
  return 0.5f * x * (1.0f + tanhf(0.7978845608f * (x + 0.044715f * x * x * x)));
}

// ---------------------------------------------------------------- activations
// Shared memory (per activation row b, per 256-column super-block sb), laid out so
// that each lane reads everything one chunk needs with a few 16-byte loads:
//   brec[((b*nsb + sb)*3 + dg)*256 + tig*64 + j*8]  8 bytes: digit plane dg of 32-block j
//                                                   at k = 4tig..4tig+3 | 16+4tig..16+4tig+3
//   sxs[b*nsb + sb]                                 digit scale of the super-block
// per MMA pair m (activation rows 2m, 2m+1 -> D columns 0..5):
//   ds32[((m*nsb + sb)*4 + tig)*8 + j]   int2: digit sums over 32-block j of D columns 2tig, 2tig+1
//   ds16[((m*nsb + sb)*4 + tig)*16 + i]  int2: the same over 16-run i
// and a 128-byte zero area that lanes without a live column read.
struct G2Smem {
  uint8_t *brec;
  float *sxs;
  int2 *ds32, *ds16;
  uint32_t zero_off;
};
__host__ __device__ inline size_t g2_smem_bytes(int nb, int cols) {
  const int nm = (nb + 1) / 2, nsb = cols / 256;
  return (size_t)nb * nsb * 768 + 128 + (size_t)nb * nsb * 4 + 16 + (size_t)nm * nsb * 256 + (size_t)nm * nsb * 512 + 64;
}
__device__ __forceinline__ G2Smem g2_carve(uint8_t *smem, int NB, int cols) {
  const int nm = (NB + 1) / 2, nsb = cols / 256;
  G2Smem S;
  S.brec = smem;
  S.zero_off = (uint32_t)NB * nsb * 768;
  size_t o = S.zero_off + 128;
  S.sxs = reinterpret_cast<float *>(smem + o);
  o += (size_t)NB * nsb * 4;
  o = (o + 15) & ~(size_t)15;
  S.ds32 = reinterpret_cast<int2 *>(smem + o);
  o += (size_t)nm * nsb * 256;
  S.ds16 = reinterpret_cast<int2 *>(smem + o);
  return S;
}

// Per-lane constants: where the lane's B records live, and which (activation
// row, digit weight) its two D columns n0 = 2tig, n1 = 2tig+1 carry per pair m.
struct G2Lane {
  uint32_t boff[2], bstride[2];  // byte offset of super-block 0 and per-super-block stride
  float w0[2], w1[2];            // digit weight of column n0 / n1 (0 when the column is unused)
  int bat0[2], bat1[2];          // activation row of column n0 / n1, or -1
};
template <int NB>
__device__ __forceinline__ G2Lane g2_lane(int grp, int tig, int nsb, uint32_t zero_off) {
  G2Lane L;
#pragma unroll
  for (int m = 0; m < 2; m++) {
    const int b = 2 * m + grp / 3, dg = grp % 3;
    const bool live = grp < 6 && b < NB;
    L.boff[m] = live ? (uint32_t)(((b * nsb) * 3 + dg) * 256 + tig * 64) : zero_off;
    L.bstride[m] = live ? 768u : 0u;
    const int n0 = 2 * tig, n1 = 2 * tig + 1;
    const int b0 = 2 * m + n0 / 3, b1 = 2 * m + n1 / 3;
    L.bat0[m] = (n0 < 6 && b0 < NB) ? b0 : -1;
    L.bat1[m] = (n1 < 6 && b1 < NB) ? b1 : -1;
    const int d0 = n0 % 3, d1 = n1 % 3;
    L.w0[m] = L.bat0[m] < 0 ? 0.f : d0 == 0 ? 1.f : d0 == 1 ? 1.f / 254.f : 1.f / 64516.f;
    L.w1[m] = L.bat1[m] < 0 ? 0.f : d1 == 0 ? 1.f : d1 == 1 ? 1.f / 254.f : 1.f / 64516.f;
  }
  return L;
}

// Thread-block cluster helpers (distributed shared memory).
constexpr int G2_CLUSTER = 8;
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Store one 32-bit word at the same shared-memory offset of every CTA of the cluster.
__device__ __forceinline__ void st_cluster_all(const void *local, uint32_t v) {
  const uint32_t la = (uint32_t)__cvta_generic_to_shared(local);
#pragma unroll
  for (int c = 0; c < G2_CLUSTER; c++) {
    uint32_t ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(la), "r"(c));
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(ra), "r"(v) : "memory");
  }
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Digitise NB activation rows (optionally RMS-normalised) into the shared memory
// of every CTA of the cluster: CTA c of the cluster handles the super-blocks
// sb = c (mod 8), one warp per super-block. Lane l takes the 4 consecutive
// columns 4(l%8).. of 32-blocks j = l/8 and j+4, packs each digit plane of the
// quad into one 32-bit word, and the digit sums of each 16-run / 32-block are
// formed from the packed words with dp4a and lane shuffles.
template <int NB>
__device__ __forceinline__ void g2_digitise(const Gemv2Args &a, const G2Smem &S, const float *inv, int warp, int lane) {
  const int nsb = a.cols >> 8;
  const int crank = (int)cluster_rank();
  const int q8 = lane & 7;                 // column quad within the 32-block
  const int tg = q8 & 3, hi = q8 >> 2;    // record lane (tig) and half (k < 16 or k >= 16)
  for (int sb = crank + G2_CLUSTER * warp; sb < nsb; sb += G2_CLUSTER * G2_WARPS) {
#pragma unroll
    for (int b = 0; b < NB; b++) {
      float4 v[2];
      float amax = 0.f;
#pragma unroll
      for (int p = 0; p < 2; p++) {
        const int j = (lane >> 3) + 4 * p;
        const int col = 256 * sb + 32 * j + 4 * q8;
        v[p] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (b < a.batch) {
          v[p] = *reinterpret_cast<const float4 *>(a.x + (int64_t)b * a.ldx + col);
          if (a.norm_w) {
            const float4 w = __ldg(reinterpret_cast<const float4 *>(a.norm_w + col));
            const float iv = inv[b];
            v[p] = make_float4(v[p].x * iv * w.x, v[p].y * iv * w.y, v[p].z * iv * w.z, v[p].w * iv * w.w);
          }
        }
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[p].x), fabsf(v[p].y)), fmaxf(fabsf(v[p].z), fabsf(v[p].w))));
      }
      amax = warp_max(amax);
      const float sc = amax > 0.f ? 127.f / amax : 0.f;
      if (lane == 0) st_cluster_all(S.sxs + b * nsb + sb, __float_as_uint(amax > 0.f ? amax / 127.f : 0.f));
      const uint8_t *rec = S.brec + (size_t)((b * nsb + sb) * 3) * 256 + tg * 64 + hi * 4;
      const int m = b >> 1, q = b & 1;
#pragma unroll
      for (int p = 0; p < 2; p++) {
        const int j = (lane >> 3) + 4 * p;
        const float xs[4] = {v[p].x, v[p].y, v[p].z, v[p].w};
        uint32_t pk[3] = {0u, 0u, 0u};
#pragma unroll
        for (int e = 0; e < 4; e++) {
          uint32_t da, db, dc;
          digits254(xs[e] * sc, da, db, dc);
          pk[0] |= da << (8 * e);
          pk[1] |= db << (8 * e);
          pk[2] |= dc << (8 * e);
        }
#pragma unroll
        for (int dg = 0; dg < 3; dg++) {
          st_cluster_all(rec + dg * 256 + j * 8, pk[dg]);
          // 16-run sum over the 4 quads (lanes differing in bits 0,1), 32-block sum adds bit 2
          int s16 = __dp4a((int)pk[dg], 0x01010101, 0);
          s16 += __shfl_xor_sync(0xffffffffu, s16, 1);
          s16 += __shfl_xor_sync(0xffffffffu, s16, 2);
          const int s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 4);
          // column n = 3q + dg of pair m sits at tig n/2, component n%2
          const int n = 3 * q + dg, tgn = n >> 1, pos = n & 1;
          if ((q8 & 3) == 0) {
            const int i = 2 * j + hi;  // 16-run index
            st_cluster_all(reinterpret_cast<int *>(S.ds16 + ((size_t)(m * nsb + sb) * 4 + tgn) * 16 + i) + pos, (uint32_t)s16);
          }
          if (q8 == 0) st_cluster_all(reinterpret_cast<int *>(S.ds32 + ((size_t)(m * nsb + sb) * 4 + tgn) * 8 + j) + pos, (uint32_t)s32);
        }
      }
    }
  }
}

// ------------------------------------------------------------------ Q4_K

struct Q4KRegs {
  uint4 qs[4];
  uint4 h0, h1;
};
__device__ __forceinline__ void q4k_load(const uint8_t *c, int lane, Q4KRegs &r) {
#pragma unroll
  for (int g = 0; g < 4; g++) r.qs[g] = ldg_stream(c + 512 * g + 16 * lane);
  const int grp = lane >> 2;
  r.h0 = ldg_stream(c + 2048 + 16 * grp);
  r.h1 = ldg_stream(c + 2048 + 16 * (grp + 8));
}

// Integer accumulators of one chunk for pair m: rows r (grp / grp+8) x columns (n0 / n1).
struct Q4KAcc {
  int I[2][2], M[2][2];
};

template <int NB>
__device__ __forceinline__ void q4k_compute(const Q4KRegs &r, int kb, const G2Smem &S, int nsb, const G2Lane &L,
                                            float (&acc)[NB][2]) {
  constexpr int NM = (NB + 1) / 2;
  const int tig = threadIdx.x & 3;
  const uint32_t M4 = 0x0F0F0F0Fu;
  // the 6-bit scale/min fields of both rows, gathered four per word
  const uint32_t sc_lo0 = r.h0.y & 0x3F3F3F3Fu, mn_lo0 = r.h0.z & 0x3F3F3F3Fu;
  const uint32_t sc_hi0 = (r.h0.w & M4) | ((r.h0.y >> 2) & 0x30303030u);
  const uint32_t mn_hi0 = ((r.h0.w >> 4) & M4) | ((r.h0.z >> 2) & 0x30303030u);
  const uint32_t sc_lo1 = r.h1.y & 0x3F3F3F3Fu, mn_lo1 = r.h1.z & 0x3F3F3F3Fu;
  const uint32_t sc_hi1 = (r.h1.w & M4) | ((r.h1.y >> 2) & 0x30303030u);
  const uint32_t mn_hi1 = ((r.h1.w >> 4) & M4) | ((r.h1.z >> 2) & 0x30303030u);
  int I[NM][2][2], Mn[NM][2][2];
  uint4 B[NM][4];
  int4 DS[NM][4];
#pragma unroll
  for (int m = 0; m < NM; m++) {
    const uint4 *bp = reinterpret_cast<const uint4 *>(S.brec + L.boff[m] + (uint32_t)kb * L.bstride[m]);
    const int4 *dp = reinterpret_cast<const int4 *>(S.ds32 + ((size_t)(m * nsb + kb) * 4 + tig) * 8);
#pragma unroll
    for (int i = 0; i < 4; i++) { B[m][i] = bp[i]; DS[m][i] = dp[i]; }
    I[m][0][0] = I[m][0][1] = I[m][1][0] = I[m][1][1] = 0;
    Mn[m][0][0] = Mn[m][0][1] = Mn[m][1][0] = Mn[m][1][1] = 0;
  }
#pragma unroll
  for (int g = 0; g < 4; g++) {
    const uint32_t w[4] = {r.qs[g].x, r.qs[g].y, r.qs[g].z, r.qs[g].w};
#pragma unroll
    for (int half = 0; half < 2; half++) {
      const int s = 2 * g + half;
      const uint32_t aa[4] = {half ? (w[0] >> 4) & M4 : w[0] & M4, half ? (w[1] >> 4) & M4 : w[1] & M4,
                              half ? (w[2] >> 4) & M4 : w[2] & M4, half ? (w[3] >> 4) & M4 : w[3] & M4};
      const int sc0 = ubyte(s < 4 ? sc_lo0 : sc_hi0, s & 3), mn0 = ubyte(s < 4 ? mn_lo0 : mn_hi0, s & 3);
      const int sc1 = ubyte(s < 4 ? sc_lo1 : sc_hi1, s & 3), mn1 = ubyte(s < 4 ? mn_lo1 : mn_hi1, s & 3);
#pragma unroll
      for (int m = 0; m < NM; m++) {
        const uint4 bq = B[m][s >> 1];
        int D[4];
        mma_k32(D, aa, (s & 1) ? bq.z : bq.x, (s & 1) ? bq.w : bq.y);
        const int4 dq = DS[m][s >> 1];
        const int dx = (s & 1) ? dq.z : dq.x, dy = (s & 1) ? dq.w : dq.y;
        // |D| <= 32*15*127 = 60960; x sc <= 63 and 8 sub-blocks: < 3.1e7. |dsum| <= 4064; x mn x 8 < 2.1e6.
        I[m][0][0] += sc0 * D[0];
        I[m][0][1] += sc0 * D[1];
        I[m][1][0] += sc1 * D[2];
        I[m][1][1] += sc1 * D[3];
        Mn[m][0][0] += mn0 * dx;
        Mn[m][0][1] += mn0 * dy;
        Mn[m][1][0] += mn1 * dx;
        Mn[m][1][1] += mn1 * dy;
      }
    }
  }
  const float d[2] = {h2f(r.h0.x), h2f(r.h1.x)}, dm[2] = {h2f(r.h0.x >> 16), h2f(r.h1.x >> 16)};
#pragma unroll
  for (int m = 0; m < NM; m++) {
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const float v0 = d[i] * (float)I[m][i][0] - dm[i] * (float)Mn[m][i][0];
      const float v1 = d[i] * (float)I[m][i][1] - dm[i] * (float)Mn[m][i][1];
      if constexpr (NB == 1) {
        const float sx = S.sxs[kb];
        acc[0][i] = fmaf(sx, fmaf(L.w0[0], v0, L.w1[0] * v1), acc[0][i]);
      } else {
#pragma unroll
        for (int b = 0; b < NB; b++) {
          if (L.bat0[m] == b) acc[b][i] = fmaf(L.w0[m] * S.sxs[b * nsb + kb], v0, acc[b][i]);
          if (L.bat1[m] == b) acc[b][i] = fmaf(L.w1[m] * S.sxs[b * nsb + kb], v1, acc[b][i]);
        }
      }
    }
  }
}

// ------------------------------------------------------------------ Q6_K

struct Q6KRegs {
  uint4 ql[4], qh[2], s0, s1;
  uint32_t d;  // fp16 d of rows grp (low half) and grp+8 (high half)
};
__device__ __forceinline__ void q6k_load(const uint8_t *c, int lane, Q6KRegs &r) {
#pragma unroll
  for (int k = 0; k < 4; k++) r.ql[k] = ldg_stream(c + 512 * k + 16 * lane);
  r.qh[0] = ldg_stream(c + 2048 + 16 * lane);
  r.qh[1] = ldg_stream(c + 2048 + 512 + 16 * lane);
  const int grp = lane >> 2;
  r.s0 = ldg_stream(c + 3072 + 16 * grp);
  r.s1 = ldg_stream(c + 3072 + 16 * (grp + 8));
  r.d = ldg_u16(c + 3328 + 2 * grp) | (ldg_u16(c + 3328 + 2 * (grp + 8)) << 16);
}

template <int NB>
__device__ __forceinline__ void q6k_compute(const Q6KRegs &r, int kb, const G2Smem &S, int nsb, const G2Lane &L,
                                            float (&acc)[NB][2]) {
  constexpr int NM = (NB + 1) / 2;
  const int tig = threadIdx.x & 3;
  const uint32_t M4 = 0x0F0F0F0Fu, T3 = 0x03030303u;
  const uint32_t sw0[4] = {r.s0.x, r.s0.y, r.s0.z, r.s0.w}, sw1[4] = {r.s1.x, r.s1.y, r.s1.z, r.s1.w};
  int I[NM][2][2];
  uint4 B[NM][4];
#pragma unroll
  for (int m = 0; m < NM; m++) {
    const uint4 *bp = reinterpret_cast<const uint4 *>(S.brec + L.boff[m] + (uint32_t)kb * L.bstride[m]);
#pragma unroll
    for (int i = 0; i < 4; i++) B[m][i] = bp[i];
    I[m][0][0] = I[m][0][1] = I[m][1][0] = I[m][1][1] = 0;
  }
  const int4 *dsp = reinterpret_cast<const int4 *>(S.ds16 + ((size_t)kb * 4 + tig) * 16);
#pragma unroll
  for (int seg = 0; seg < 2; seg++) {
    const uint32_t hw[4] = {r.qh[seg].x, r.qh[seg].y, r.qh[seg].z, r.qh[seg].w};
#pragma unroll
    for (int quarter = 0; quarter < 4; quarter++) {
      const int qp = quarter & 1, nib = quarter >> 1;
      const uint4 lw = r.ql[2 * seg + qp];
      const uint32_t l[4] = {lw.x, lw.y, lw.z, lw.w};
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int s = 8 * seg + 2 * quarter + h;  // sub-block of 16 values; 32-block s/2, half h
        const uint32_t a0 = ((l[2 * h] >> (4 * nib)) & M4) | (((hw[2 * h] >> (2 * quarter)) & T3) << 4);
        const uint32_t a1 = ((l[2 * h + 1] >> (4 * nib)) & M4) | (((hw[2 * h + 1] >> (2 * quarter)) & T3) << 4);
        const int sc0 = sbyte(sw0[s >> 2], s & 3), sc1 = sbyte(sw1[s >> 2], s & 3);
#pragma unroll
        for (int m = 0; m < NM; m++) {
          const uint4 bq = B[m][s >> 2];
          const int j = s >> 1;  // 32-block within the super-block
          const uint32_t b0 = (j & 1) ? (h ? bq.w : bq.z) : (h ? bq.y : bq.x);
          int D[4];
          mma_k16(D, a0, a1, b0);
          const int4 dq = (m == 0 ? dsp : reinterpret_cast<const int4 *>(S.ds16 + ((size_t)(m * nsb + kb) * 4 + tig) * 16))[s >> 1];
          const int dx = (s & 1) ? dq.z : dq.x, dy = (s & 1) ? dq.w : dq.y;
          // |D - 32*dsum| <= 16*32*127 = 65024; x |sc| <= 128 and 16 sub-blocks: < 1.4e8.
          I[m][0][0] += sc0 * (D[0] - 32 * dx);
          I[m][0][1] += sc0 * (D[1] - 32 * dy);
          I[m][1][0] += sc1 * (D[2] - 32 * dx);
          I[m][1][1] += sc1 * (D[3] - 32 * dy);
        }
      }
    }
  }
  const float d[2] = {h2f(r.d), h2f(r.d >> 16)};
#pragma unroll
  for (int m = 0; m < NM; m++) {
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const float v0 = d[i] * (float)I[m][i][0], v1 = d[i] * (float)I[m][i][1];
      if constexpr (NB == 1) {
        acc[0][i] = fmaf(S.sxs[kb], fmaf(L.w0[0], v0, L.w1[0] * v1), acc[0][i]);
      } else {
#pragma unroll
        for (int b = 0; b < NB; b++) {
          if (L.bat0[m] == b) acc[b][i] = fmaf(L.w0[m] * S.sxs[b * nsb + kb], v0, acc[b][i]);
          if (L.bat1[m] == b) acc[b][i] = fmaf(L.w1[m] * S.sxs[b * nsb + kb], v1, acc[b][i]);
        }
      }
    }
  }
}

// ------------------------------------------------------------------ kernel

template <int T> struct TileOps;
template <> struct TileOps<Q4_K> {
  using Regs = Q4KRegs;
  static constexpr int CB = 2304;
  static __device__ __forceinline__ void load(const uint8_t *c, int lane, Regs &r) { q4k_load(c, lane, r); }
  template <int NB>
  static __device__ __forceinline__ void compute(const Regs &r, int kb, const G2Smem &S, int cols, const G2Lane &L,
                                                 float (&acc)[NB][2]) { q4k_compute<NB>(r, kb, S, cols >> 8, L, acc); }
};
template <> struct TileOps<Q6_K> {
  using Regs = Q6KRegs;
  static constexpr int CB = 3360;
  static __device__ __forceinline__ void load(const uint8_t *c, int lane, Regs &r) { q6k_load(c, lane, r); }
  template <int NB>
  static __device__ __forceinline__ void compute(const Regs &r, int kb, const G2Smem &S, int cols, const G2Lane &L,
                                                 float (&acc)[NB][2]) { q6k_compute<NB>(r, kb, S, cols >> 8, L, acc); }
};

// Units are split over W workers as q = U / W each, the first rem = U % W
// workers taking one more: worker i starts at i*q + min(i, rem).
struct Split {
  int q, rem, thr;  // thr = rem * (q + 1): first unit owned by a q-sized worker
  __device__ __forceinline__ int start(int i) const { return i * q + (i < rem ? i : rem); }
  __device__ __forceinline__ int worker_of(int u) const { return u < thr ? u / (q + 1) : rem + (u - thr) / q; }
};

// Epilogue for one finished tile: lane 4r (+tig 0) holds rows r and r+8 for each activation row.
template <int NB>
__device__ __forceinline__ void g2_store(const Gemv2Args &a, int t, int grp, const float (&v)[NB][2]) {
#pragma unroll
  for (int b = 0; b < NB; b++) {
    if (b >= a.batch) continue;
    if (a.epi == EPI_GLU_SILU || a.epi == EPI_GLU_GELU) {
      // tile rows 0..7 are gate rows, 8..15 the matching up rows
      if (t * 16 + grp < a.rows) {
        const float g = v[b][0], u = v[b][1];
        a.y[(int64_t)b * a.ldy + t * 8 + grp] = (a.epi == EPI_GLU_SILU ? g2_silu(g) : g2_gelu(g)) * u;
      }
      continue;
    }
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const int row = t * 16 + grp + 8 * i;
      if (row >= a.rows) continue;
      float val = v[b][i];
      if (a.bias) val += __ldg(a.bias + row);
      float *dst = a.y + (int64_t)b * a.ldy + row;
      if (a.epi == EPI_ADD) *dst = __ldcg(dst) + val;  // through L2, so that no stale line stays in L1
      else if (a.epi == EPI_SILU) *dst = g2_silu(val);
      else *dst = val;
    }
  }
}

template <int T, int NB>
__global__ void __launch_bounds__(G2_WARPS * 32) gemv2_kernel(const Gemv2Args a) {
  using Ops = TileOps<T>;
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float s_norm[G2_WARPS][NB];
  __shared__ float s_inv[NB];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, grp = lane >> 2, tig = lane & 3;
  // workers: the first min(warps, units) warps, so that every worker owns at least one unit
  const int U = a.tiles * a.nkb, Wall = gridDim.x * G2_WARPS;
  const int W = Wall < U ? Wall : U;
  Split sp;
  sp.q = U / W;
  sp.rem = U - sp.q * W;
  sp.thr = sp.rem * (sp.q + 1);
  const int wid = blockIdx.x * G2_WARPS + warp;
  const int u0 = wid < W ? sp.start(wid) : U, u1 = wid < W ? sp.start(wid + 1) : U;

  // prologue: the first chunk of this warp (weights only, independent of earlier kernels)
  typename Ops::Regs ra, rb;
  const uint8_t *wp = a.w + (size_t)u0 * Ops::CB;  // chunk of unit cu
  if (u0 < u1) Ops::load(wp, lane, ra);
  // The dependents are released only after this kernel's own wait: then at most the next
  // kernel is resident beside this one, and no kernel two launches later can find
  // residual-stream lines in L1 that this kernel's norm prologue read and that the
  // next kernel updated.
  pdl_wait();
  pdl_launch_dependents();

  const G2Smem S = g2_carve(smem, NB, a.cols);
  // the zero record read by lanes without a live MMA column (digit-sum entries of
  // unused columns are never written: they only meet zero weights, and an int
  // converted to float is always finite)
  if (tid < 32) reinterpret_cast<uint32_t *>(S.brec + S.zero_off)[tid] = 0u;
  if (a.norm_w) {
#pragma unroll
    for (int b = 0; b < NB; b++) {
      float s = 0.f;
      if (b < a.batch) {
        const float4 *xr = reinterpret_cast<const float4 *>(a.x + (int64_t)b * a.ldx);
        for (int c = tid; c < (a.cols >> 2); c += blockDim.x) {
          const float4 v = xr[c];
          s = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, s))));
        }
      }
      s = warp_sum(s);
      if (lane == 0) s_norm[warp][b] = s;
    }
    __syncthreads();
    if (tid < NB) {
      float t = 0.f;
      for (int w = 0; w < G2_WARPS; w++) t += s_norm[w][tid];
      s_inv[tid] = rsqrtf(t / (float)a.cols + a.eps);
    }
    __syncthreads();
  }
  // every CTA of the cluster must be running before remote stores reach it
  cluster_sync();
  g2_digitise<NB>(a, S, s_inv, warp, lane);
  cluster_sync();
  if (u0 >= u1) return;
  const G2Lane L = g2_lane<NB>(grp, tig, a.cols >> 8, S.zero_off);

  int cu = u0;
  bool in_b = false;  // which register set holds chunk cu
  const int t_first = u0 / a.nkb, t_last = (u1 - 1) / a.nkb;
  for (int t = t_first; t <= t_last; t++) {
    const int tlo = t * a.nkb, thi = tlo + a.nkb;
    const int seg_hi = u1 < thi ? u1 : thi;
    float acc[NB][2];
#pragma unroll
    for (int b = 0; b < NB; b++) acc[b][0] = acc[b][1] = 0.f;
    while (cu < seg_hi) {
      const int kb = cu - tlo;
      const bool more = cu + 1 < u1;
      wp += Ops::CB;
      if (!in_b) {
        if (more) Ops::load(wp, lane, rb);
        Ops::template compute<NB>(ra, kb, S, a.cols, L, acc);
      } else {
        if (more) Ops::load(wp, lane, ra);
        Ops::template compute<NB>(rb, kb, S, a.cols, L, acc);
      }
      in_b = !in_b;
      cu++;
    }
    // sum the four lanes of each row group: lane tig 0 then holds rows grp, grp+8
#pragma unroll
    for (int b = 0; b < NB; b++)
#pragma unroll
      for (int i = 0; i < 2; i++) {
        acc[b][i] += __shfl_xor_sync(0xffffffffu, acc[b][i], 1);
        acc[b][i] += __shfl_xor_sync(0xffffffffu, acc[b][i], 2);
      }
    const int seg_lo = u0 > tlo ? u0 : tlo;
    if (seg_lo == tlo && seg_hi == thi) {
      if (tig == 0) g2_store<NB>(a, t, grp, acc);
      continue;
    }
    // split tile: publish the partial, the last arriving worker finishes the tile
    const int w0 = sp.worker_of(tlo), w1 = sp.worker_of(thi - 1);
    const int slot = wid - w0, count = w1 - w0 + 1;
    float *pt = a.part + (size_t)t * a.maxc * 16 * NB;
    if (tig == 0) {
#pragma unroll
      for (int b = 0; b < NB; b++) {
        pt[(size_t)slot * 16 * NB + b * 16 + grp] = acc[b][0];
        pt[(size_t)slot * 16 * NB + b * 16 + grp + 8] = acc[b][1];
      }
    }
    __threadfence();
    __syncwarp();
    unsigned prev = 0;
    if (lane == 0) prev = atomicAdd(a.tile_ctr + t, 1u);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev == (unsigned)(count - 1)) {
      __threadfence();
      float v[NB][2];
#pragma unroll
      for (int b = 0; b < NB; b++) {
        v[b][0] = v[b][1] = 0.f;
        for (int j = 0; j < count; j++) {
          v[b][0] += __ldcg(pt + (size_t)j * 16 * NB + b * 16 + grp);
          v[b][1] += __ldcg(pt + (size_t)j * 16 * NB + b * 16 + grp + 8);
        }
      }
      if (tig == 0) g2_store<NB>(a, t, grp, v);
      if (lane == 0) a.tile_ctr[t] = 0u;
    }
  }
}

// Partial slots one tile may need: workers touching a tile of nkb units when each
// worker owns at least floor(U/W) units.
inline int gemv2_maxc(int tiles, int nkb, long long workers) {
  const long long U = (long long)tiles * nkb;
  if (workers >= U) return nkb;
  const long long per = U / workers;
  long long c = (nkb + per - 1) / per + 1;
  if (c > nkb) c = nkb;
  return (int)(c < 1 ? 1 : c);
}

template <int T, int NB>
cudaError_t launch_gemv2_cfg(const Gemv2Args &a, cudaStream_t s, bool pdl, int sm_count) {
  (void)sm_count;
  const size_t smem = g2_smem_bytes(NB, a.cols);
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(G2_WARPS * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = G2_CLUSTER;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  static int clusters = -1;
  static size_t occ_smem = 0;
  if (clusters < 0 || occ_smem != smem) {
    cudaFuncSetAttribute(gemv2_kernel<T, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    cfg.gridDim = dim3(G2_CLUSTER);
    if (cudaOccupancyMaxActiveClusters(&clusters, gemv2_kernel<T, NB>, &cfg) != cudaSuccess || clusters < 1) clusters = 1;
    occ_smem = smem;
  }
  long long grid = (long long)clusters * G2_CLUSTER;
  const long long U = (long long)a.tiles * a.nkb;
  const long long maxgrid = (U + G2_WARPS - 1) / G2_WARPS;  // at least one unit per warp
  if (grid > maxgrid) grid = (maxgrid + G2_CLUSTER - 1) / G2_CLUSTER * G2_CLUSTER;
  if (grid < G2_CLUSTER) grid = G2_CLUSTER;
  cfg.gridDim = dim3((unsigned)grid);
  return cudaLaunchKernelEx(&cfg, gemv2_kernel<T, NB>, a);
}

template <int T>
cudaError_t launch_gemv2_type(const Gemv2Args &a, cudaStream_t s, bool pdl, int sm_count) {
  if (a.batch == 1) return launch_gemv2_cfg<T, 1>(a, s, pdl, sm_count);
  if (a.batch == 2) return launch_gemv2_cfg<T, 2>(a, s, pdl, sm_count);
  return launch_gemv2_cfg<T, 4>(a, s, pdl, sm_count);
}

}  // namespace wgd
