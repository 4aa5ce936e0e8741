// Prompt-batch GEMM on the 5th-generation tensor cores (tcgen05 + tensor
// memory) for Q4_K and Q6_K weights in the tile-16 layout (tile.cuh):
//   y[b][row] (op)= sum_k W[row][k] * x[b][k],   b < batch <= 128,
// the operation of the reference's matmul shader for a prompt batch
// (shaders.ts matmul over `batchSize` rows, driven by engine.ts:217-251).
//
// Exactness. A Q4_K weight is d*sc_j*q - dmin*mn_j (super-block scales d, dmin;
// 6-bit sub-block scale/min sc_j, mn_j; 4-bit quant q). The tensor core gets
//   A = sc_j*q            an integer <= 945: exact in f16,
//   B = x_hi + x_lo       the activation as two f16 terms (x_lo = x - x_hi),
// so one f32 accumulator R = sum_k A*(x_hi + x_lo) per 256-column super-block
// carries the activation to ~2^-22 and the weights exactly. A second small MMA
// gives Mn = sum_j mn_j * S_j with S_j = sum of x over sub-block j (also split
// hi/lo), and the epilogue applies the super-block scales in fp32:
//   y += d*R - dmin*Mn.
// Q6_K (d*sc*(q-32), no mins): A is two exact f16 terms (see role_dequant<Q6_K>),
// four MMAs per K-step (A_hi, A_lo against x_hi, x_lo), y += d*R.
// Each activation row is scaled by a power of two first (max |x| in [512, 1024))
// so that x_hi, x_lo and S stay inside the f16 range; the epilogue undoes it.
//
// Data flow per CTA (one CTA per SM, a contiguous range of (M-tile, super-block)
// units, M-tile = 128 weight rows = 8 tiles of 16):
//   raw producer warp : bulk copies of the unit's 8 tile chunks -> raw ring (2)
//   B producer warp   : bulk copy of the prepared activation panel of each
//                       64-column stage (x_hi | x_lo [| S]) -> stage ring
//   8 dequant warps   : raw quants -> A = sc*q (f16, K-major core matrices) in
//                       the stage, plus the 128 x 16 "mins" operand on the last
//                       stage of a unit
//   MMA warp          : 4 stages x 4 K-steps x (hi, lo) tcgen05.mma M128 N<=128
//                       K16 into R[unit & 1], then the mins MMA into Mn; commits
//                       release the stage and publish the unit
//   4 epilogue warps  : TMEM lanes 32q..32q+31 (one weight row per thread):
//                       Y = Y + d*R - dmin*Mn kept in tensor memory across the
//                       unit range; at the end of an M-tile segment the rows are
//                       written out (bias / residual add / SiLU / gated
//                       activations), or as a partial that the CTA arriving
//                       last for that M-tile sums in CTA order (deterministic).
// Tensor memory columns: [0,N) R0, [N,2N) R1, [2N,3N) Mn, [3N,4N) Y.
// Within a CTA's M-tile segment the super-blocks start at a per-CTA rotation, so
// that CTAs running at the same time read different parts of the panel.
// Every mbarrier wait is bounded (2 s of globaltimer); a wait that runs out
// sets *status = 1 and the CTA winds down (copies and MMAs in flight are
// waited for, tensor memory is freed).
#include <cuda_fp16.h>

#include "kernels.h"
#include "tile.cuh"
#include "umma.cuh"

namespace wgd {
namespace {

using namespace tc;

constexpr int TC_M = 128;                            // weight rows per M-tile
constexpr int TC_TILES = TC_M / TILE_ROWS;           // tiles per M-tile
constexpr int TC_DQ = 8;                             // dequant warps 0..7 (one tile each)
constexpr int TC_EPI0 = 8;                           // epilogue warps 8..11: TMEM lane quarters 0..3
constexpr int TC_EPIW = 4;
constexpr int TC_RAWW = 12, TC_BW = 13, TC_MMAW = 14;  // single-lane roles (the MMA warp also owns the tensor memory)
// Registers are handed out per group of 4 warps: 15 warps cost 16 warps' worth, at
// most 128 per thread.
constexpr int TC_THREADS = 15 * 32;
constexpr int TC_A_BYTES = TC_M * 64 * 2;            // A of one 64-column stage
constexpr int TC_AMIN_BYTES = TC_M * 16 * 2;         // mins operand
constexpr int TC_HDR = 1024;                         // barriers, words, column scales
constexpr int TC_MAXST = 8;
constexpr int TC_SMEM_MAX = 232448;                  // 227 KB opt-in
constexpr uint64_t TC_TIMEOUT_NS = 2000000000ull;

// Panel (prepared activations) per super-block: 4 stages of [hi N x 64][lo N x 64]
// f16, then the sums operand [N x 16] f16; after all super-blocks, N f32 column scales.
__host__ __device__ inline size_t panel_kb_bytes(int N) { return (size_t)N * 1056; }
// Per weight type: tile chunk bytes, and the stage layout after A: Q4_K keeps the
// 128 x 16 mins operand there, Q6_K the low part of its two-term A.
template <int T> struct TcType;
template <> struct TcType<Q4_K> {
  static constexpr int CHUNK = 2304, A2 = TC_AMIN_BYTES;
  static constexpr bool MINS = true;
};
template <> struct TcType<Q6_K> {
  static constexpr int CHUNK = 3360, A2 = TC_A_BYTES;
  static constexpr bool MINS = false;
};
__host__ __device__ inline int tc_chunk(int type) { return type == Q4_K ? 2304 : 3360; }
__host__ __device__ inline int raw_bytes(int type) { return TC_TILES * tc_chunk(type); }
__host__ __device__ inline uint32_t stage_bytes(int type, int N) {
  return type == Q4_K ? (uint32_t)(TC_A_BYTES + TC_AMIN_BYTES + N * 288) : (uint32_t)(2 * TC_A_BYTES + N * 256);
}

struct TcArgs {
  const uint8_t *w;
  int rows, cols, nkb, tiles, mtiles;
  const uint8_t *panel;
  int N, batch;
  float *y;
  int ldy;
  const float *bias;
  int epi;
  float *part;
  unsigned *ctr;
  int *status;
  int nstage;
  uint32_t sbytes, tmem_cols;
  int q, rem, thr;  // units split: CTA c owns [c*q + min(c, rem), +q (+1 if c < rem))
};

__device__ __forceinline__ int unit_start(const TcArgs &a, int c) { return c * a.q + (c < a.rem ? c : a.rem); }
__device__ __forceinline__ int unit_owner(const TcArgs &a, int u) {
  return u < a.thr ? u / (a.q + 1) : a.rem + (u - a.thr) / a.q;
}

// The unit at position U of this CTA's range [u0, u1): the range is cut into M-tile
// segments, and each segment's super-blocks are visited from a per-CTA rotation on
// (kb0 + (j + rot) mod len), so that CTAs running at the same time read different
// parts of the activation panel. j is the position inside the segment.
struct UnitPos {
  int mt, kb, j, len;
};
__device__ __forceinline__ UnitPos unit_pos(const TcArgs &a, int u0, int u1, int U) {
  UnitPos p;
  p.mt = U / a.nkb;
  const int seg0 = max(u0, p.mt * a.nkb), seg1 = min(u1, (p.mt + 1) * a.nkb);
  p.len = seg1 - seg0;
  p.j = U - seg0;
  const int rot = (int)((blockIdx.x * 7u) % (unsigned)p.len);
  p.kb = seg0 - p.mt * a.nkb + (p.j + rot) % p.len;
  return p;
}

__device__ bool tc_wait(uint64_t *b, unsigned par, volatile int *stop, int *status) {
  if (mbar_test(b, par)) return true;
  const uint64_t t0 = gtime();
  while (!mbar_try_sleep(b, par, 1000000u)) {
    if (*stop) return false;
    if (gtime() - t0 > TC_TIMEOUT_NS) {
      atomicCAS(status, 0, 1);
      *stop = 1;
      return false;
    }
  }
  return true;
}
// Waits for a phase regardless of the stop flag (copies / MMAs in flight at exit).
__device__ void tc_drain(uint64_t *b, unsigned par) {
  const uint64_t t0 = gtime();
  while (!mbar_test(b, par)) {
    if (gtime() - t0 > TC_TIMEOUT_NS) break;
    __nanosleep(64);
  }
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(0u), "r"(sel));
  return r;
}
// (a & 0x000F000F) | 0x64006400: two f16 values 1024 + nibble
__device__ __forceinline__ uint32_t nib2(uint32_t a) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(0x000F000Fu), "r"(0x64006400u));
  return r;
}
__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}
__device__ __forceinline__ uint32_t h2pair(float lo, float hi) {
  return (uint32_t)__half_as_ushort(__float2half_rn(lo)) | ((uint32_t)__half_as_ushort(__float2half_rn(hi)) << 16);
}
__device__ __forceinline__ void sts64(uint8_t *p, uint32_t a, uint32_t b) {
  asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(su32(p)), "r"(a), "r"(b) : "memory");
}
__device__ __forceinline__ void sts128(uint8_t *p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(su32(p)), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ float tc_silu(float g) { return g / (1.0f + expf(-g)); }
__device__ __forceinline__ float tc_gelu(float x) {
  return 0.5f * x * (1.0f + tanhf(0.7978845608f * (x + 0.044715f * x * x * x)));
}

// The 6-bit scales (sc) and mins (mn) of sub-blocks 0..3 / 4..7 of one row as
// packed bytes, from the 12 GGUF scale bytes s0 = bytes 0..3, s1 = 4..7, s2 = 8..11.
struct Q4Scales {
  uint32_t sc_lo, sc_hi, mn_lo, mn_hi;
};
__device__ __forceinline__ Q4Scales q4_scales(uint32_t s0, uint32_t s1, uint32_t s2) {
  Q4Scales r;
  r.sc_lo = s0 & 0x3F3F3F3Fu;
  r.mn_lo = s1 & 0x3F3F3F3Fu;
  r.sc_hi = (s2 & 0x0F0F0F0Fu) | (((s0 >> 6) & 0x03030303u) << 4);
  r.mn_hi = ((s2 >> 4) & 0x0F0F0F0Fu) | (((s1 >> 6) & 0x03030303u) << 4);
  return r;
}
__device__ __forceinline__ uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xFFu; }
// (sc, sc) and (-1024 sc, -1024 sc) as f16x2
__device__ __forceinline__ void sc_pair(uint32_t sc, uint32_t &s2, uint32_t &n2) {
  const uint32_t h = __half_as_ushort(__uint2half_rn(sc));
  const uint32_t n = __half_as_ushort(__int2half_rn(-1024 * (int)sc));
  s2 = h | (h << 16);
  n2 = n | (n << 16);
}

// ------------------------------------------------------------------ roles

template <int T>
__device__ void role_raw(const TcArgs &a, uint8_t *raw, uint64_t *rawfull, uint64_t *rawempty, volatile int *stop, int u0,
                         int u1) {
  constexpr int CH = TcType<T>::CHUNK, RAW = TC_TILES * CH;
  int i = 0;
  for (int U = u0; U < u1; U++, i++) {
    const UnitPos P = unit_pos(a, u0, u1, U);
    const int mt = P.mt, kb = P.kb, r = i & 1;
    if (!tc_wait(rawempty + r, ((i >> 1) & 1) ^ 1, stop, a.status)) break;
    const int n = min(TC_TILES, a.tiles - mt * TC_TILES);
    mbar_expect_tx(rawfull + r, (unsigned)(n * CH));
    for (int t = 0; t < n; t++)
      bulk_g2s(raw + r * RAW + t * CH, a.w + ((size_t)(mt * TC_TILES + t) * a.nkb + kb) * CH, CH, rawfull + r);
  }
  for (int j = max(0, i - 2); j < i; j++) tc_drain(rawfull + (j & 1), (j >> 1) & 1);
}

template <int T>
__device__ void role_b(const TcArgs &a, uint8_t *stages, uint64_t *bfull, uint64_t *empty, volatile int *stop, int u0, int u1) {
  const int N = a.N;
  unsigned G = 0;
  for (int U = u0; U < u1; U++) {
    const int kb = unit_pos(a, u0, u1, U).kb;
    for (int g = 0; g < 4; g++, G++) {
      const int s = G % a.nstage;
      if (!tc_wait(empty + s, ((G / a.nstage) & 1) ^ 1, stop, a.status)) goto done;
      const unsigned bytes = (unsigned)(N * 256 + (TcType<T>::MINS && g == 3 ? N * 32 : 0));
      mbar_expect_tx(bfull + s, bytes);
      bulk_g2s(stages + (size_t)s * a.sbytes + TC_A_BYTES + TcType<T>::A2, a.panel + (size_t)kb * panel_kb_bytes(N) + (size_t)g * N * 256,
               bytes, bfull + s);
    }
  }
done:
  for (unsigned j = G > (unsigned)a.nstage ? G - a.nstage : 0u; j < G; j++) tc_drain(bfull + j % a.nstage, (j / a.nstage) & 1);
}

template <int T>
__device__ void role_dequant(const TcArgs &a, uint8_t *raw, uint8_t *stages, uint64_t *afull, uint64_t *empty, uint64_t *rawfull,
                             uint64_t *rawempty, volatile int *stop, int u0, int u1, int warp, int lane);

template <>
__device__ void role_dequant<Q4_K>(const TcArgs &a, uint8_t *raw, uint8_t *stages, uint64_t *afull, uint64_t *empty, uint64_t *rawfull,
                                   uint64_t *rawempty, volatile int *stop, int u0, int u1, int warp, int lane) {
  constexpr int CH = TcType<Q4_K>::CHUNK, RAW = TC_TILES * CH;
  const int grp = lane >> 2, tig = lane & 3;
  unsigned G = 0;
  int i = 0;
  for (int U = u0; U < u1; U++, i++) {
    const int mt = U / a.nkb, r = i & 1;
    bool ok = tc_wait(rawfull + r, (i >> 1) & 1, stop, a.status);
    if (!__all_sync(0xffffffffu, ok)) return;
    const bool present = mt * TC_TILES + warp < a.tiles;
    const uint8_t *chunk = raw + r * RAW + warp * CH;
    // scales of rows grp (rs 0) and grp + 8 (rs 1)
    Q4Scales S[2];
#pragma unroll
    for (int rs = 0; rs < 2; rs++) {
      const uint4 h = *reinterpret_cast<const uint4 *>(chunk + 2048 + 16 * (grp + 8 * rs));
      S[rs] = q4_scales(h.y, h.z, h.w);
    }
    for (int g = 0; g < 4; g++, G++) {
      const int s = G % a.nstage;
      ok = tc_wait(empty + s, ((G / a.nstage) & 1) ^ 1, stop, a.status);
      if (!__all_sync(0xffffffffu, ok)) return;
      uint8_t *A = stages + (size_t)s * a.sbytes;
      if (present) {
        const uint4 qv = *reinterpret_cast<const uint4 *>(chunk + g * 512 + lane * 16);
        const uint32_t W[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
        for (int rs = 0; rs < 2; rs++) {
          const uint32_t scw = g < 2 ? S[rs].sc_lo : S[rs].sc_hi;
          uint32_t sa, na, sb, nb;
          sc_pair(byte_of(scw, (2 * g) & 3), sa, na);      // sub-block 2g: low nibbles
          sc_pair(byte_of(scw, (2 * g + 1) & 3), sb, nb);  // sub-block 2g+1: high nibbles
          uint8_t *row = A + (2 * warp + rs) * 1024 + grp * 16 + (tig & 1) * 8;
#pragma unroll
          for (int part = 0; part < 2; part++) {
            const uint32_t t = prmt(W[part * 2 + rs], 0x3120u);  // bytes b0 b2 b1 b3
            const uint32_t kc = 2 * part + (tig >> 1);            // core matrix along K of k = 16 part + 4 tig
            sts64(row + kc * 128, hfma2(nib2(t), sa, na), hfma2(nib2(t >> 8), sa, na));
            sts64(row + (kc + 4) * 128, hfma2(nib2(t >> 4), sb, nb), hfma2(nib2(t >> 12), sb, nb));
          }
        }
        if (g == 3) {
          // mins operand: row grp + 8*(tig>>1), K columns 8*(tig&1) .. +7 = mn_0..mn_7
          const uint32_t mlo = (tig >> 1) ? S[1].mn_lo : S[0].mn_lo, mhi = (tig >> 1) ? S[1].mn_hi : S[0].mn_hi;
          uint32_t h[4];
#pragma unroll
          for (int p = 0; p < 4; p++) {
            const uint32_t m0 = byte_of(p < 2 ? mlo : mhi, (2 * p) & 3), m1 = byte_of(p < 2 ? mlo : mhi, (2 * p + 1) & 3);
            h[p] = (uint32_t)__half_as_ushort(__uint2half_rn(m0)) | ((uint32_t)__half_as_ushort(__uint2half_rn(m1)) << 16);
          }
          sts128(A + TC_A_BYTES + (2 * warp + (tig >> 1)) * 256 + (tig & 1) * 128 + grp * 16, h[0], h[1], h[2], h[3]);
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(afull + s);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(rawempty + r);
  }
}

// Q6_K: a weight is d*sc*(q - 32), sc an int8 per 16 columns, q 6 bits (low nibble
// in ql, two high bits in qh). sc*(q - 32) reaches 4064 in magnitude, past the
// integers f16 holds exactly, so A is written as two exact f16 terms with the
// scale split into its even part and its last bit: A_hi = (sc & ~1)*(q - 32)
// (even, <= 4096), A_lo = (sc & 1)*(q - 32); each term is one fma.rn.f16x2 from
// the f16 value 64 + q (q placed in mantissa bits 4..9 of 64.0): (64 + q)*s - 96*s.
template <>
__device__ void role_dequant<Q6_K>(const TcArgs &a, uint8_t *raw, uint8_t *stages, uint64_t *afull, uint64_t *empty, uint64_t *rawfull,
                                   uint64_t *rawempty, volatile int *stop, int u0, int u1, int warp, int lane) {
  constexpr int CH = TcType<Q6_K>::CHUNK, RAW = TC_TILES * CH;
  const int grp = lane >> 2, tig = lane & 3;
  unsigned G = 0;
  int i = 0;
  for (int U = u0; U < u1; U++, i++) {
    const int mt = U / a.nkb, r = i & 1;
    bool ok = tc_wait(rawfull + r, (i >> 1) & 1, stop, a.status);
    if (!__all_sync(0xffffffffu, ok)) return;
    const bool present = mt * TC_TILES + warp < a.tiles;
    const uint8_t *chunk = raw + r * RAW + warp * CH;
    for (int g = 0; g < 4; g++, G++) {
      const int s = G % a.nstage;
      ok = tc_wait(empty + s, ((G / a.nstage) & 1) ^ 1, stop, a.status);
      if (!__all_sync(0xffffffffu, ok)) return;
      uint8_t *A = stages + (size_t)s * a.sbytes;
      if (present) {
        // stage g = columns 64g.. of the super-block: segment g >> 1, quarters 2hq, 2hq + 1
        const int seg = g >> 1, hq = g & 1;
        const uint4 l0 = *reinterpret_cast<const uint4 *>(chunk + (2 * seg) * 512 + lane * 16);
        const uint4 l1 = *reinterpret_cast<const uint4 *>(chunk + (2 * seg + 1) * 512 + lane * 16);
        const uint4 hv = *reinterpret_cast<const uint4 *>(chunk + 2048 + seg * 512 + lane * 16);
        const uint32_t QL[2][4] = {{l0.x, l0.y, l0.z, l0.w}, {l1.x, l1.y, l1.z, l1.w}};
        const uint32_t QH[4] = {hv.x, hv.y, hv.z, hv.w};
#pragma unroll
        for (int wi = 0; wi < 4; wi++) {  // word order: (row grp, h 0), (row grp+8, h 0), (row grp, h 1), (row grp+8, h 1)
          const int h = wi >> 1, rs = wi & 1, row = grp + 8 * rs;
          uint8_t *dst = A + (2 * warp + rs) * 1024 + grp * 16 + (tig & 1) * 8;
          const uint32_t u = prmt(QH[wi], 0x3120u);  // qh bytes c0 c2 c1 c3
#pragma unroll
          for (int qp = 0; qp < 2; qp++) {
            const int quarter = 2 * hq + qp;
            const uint32_t t = prmt(QL[qp][wi], 0x3120u);  // ql bytes b0 b2 b1 b3
            // f16 64 + q of columns (4tig, 4tig+1) and (4tig+2, 4tig+3) of this 16-column run
            const uint32_t n01 = (hq ? t : t << 4) & 0x00F000F0u, n23 = (hq ? t >> 8 : t >> 4) & 0x00F000F0u;
            const uint32_t h01 = (u << (8 - 2 * quarter)) & 0x03000300u, h23 = (u >> (2 * quarter)) & 0x03000300u;
            const uint32_t x01 = n01 | h01 | 0x54005400u, x23 = n23 | h23 | 0x54005400u;
            const int sc = (int)(int8_t)chunk[3072 + 16 * row + seg * 8 + quarter * 2 + h];
            const int se = sc & ~1, so = sc & 1;
            const uint32_t she = __half_as_ushort(__int2half_rn(se)), nhe = __half_as_ushort(__int2half_rn(-96 * se));
            const uint32_t sho = __half_as_ushort(__int2half_rn(so)), nho = __half_as_ushort(__int2half_rn(-96 * so));
            const uint32_t se2 = she | (she << 16), ne2 = nhe | (nhe << 16), so2 = sho | (sho << 16), no2 = nho | (nho << 16);
            const int kc = 4 * qp + 2 * h + (tig >> 1);  // core matrix along K of k = 32qp + 16h + 4tig
            sts64(dst + kc * 128, hfma2(x01, se2, ne2), hfma2(x23, se2, ne2));
            sts64(dst + TC_A_BYTES + kc * 128, hfma2(x01, so2, no2), hfma2(x23, so2, no2));
          }
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(afull + s);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(rawempty + r);
  }
}

template <int T>
__device__ void role_mma(const TcArgs &a, uint32_t tbase, uint8_t *stages, uint64_t *bfull, uint64_t *afull, uint64_t *empty, uint64_t *accfull,
                         uint64_t *accempty, uint64_t *mnempty, uint64_t *drain, volatile int *stop, int u0, int u1) {
  const int N = a.N;
  const uint32_t idesc = idesc_f16_f32(TC_M, N);
  const uint32_t tMn = tbase + 2 * N;
  unsigned G = 0;
  int i = 0;
  for (int U = u0; U < u1; U++, i++) {
    const int b = i & 1;
    if (!tc_wait(accempty + b, ((i >> 1) & 1) ^ 1, stop, a.status)) goto done;
    tc_fence_after();
    for (int g = 0; g < 4; g++, G++) {
      const int s = G % a.nstage;
      if (!tc_wait(bfull + s, (G / a.nstage) & 1, stop, a.status) || !tc_wait(afull + s, (G / a.nstage) & 1, stop, a.status))
        goto done;
      tc_fence_after();
      const uint32_t sa = su32(stages + (size_t)s * a.sbytes), sb = sa + TC_A_BYTES + TcType<T>::A2;
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const uint64_t ad = sdesc(sa + k * 256, 128, 1024);
        mma_f16(tbase + b * N, ad, sdesc(sb + k * 256, 128, 1024), idesc, (g | k) != 0);
        mma_f16(tbase + b * N, ad, sdesc(sb + N * 128 + k * 256, 128, 1024), idesc, 1u);
        if (!TcType<T>::MINS) {  // the low term of A (Q6_K) against both activation terms
          const uint64_t al = sdesc(sa + TC_A_BYTES + k * 256, 128, 1024);
          mma_f16(tbase + b * N, al, sdesc(sb + k * 256, 128, 1024), idesc, 1u);
          mma_f16(tbase + b * N, al, sdesc(sb + N * 128 + k * 256, 128, 1024), idesc, 1u);
        }
      }
      if (TcType<T>::MINS && g == 3) {
        if (!tc_wait(mnempty, (i & 1) ^ 1, stop, a.status)) goto done;
        tc_fence_after();
        mma_f16(tMn, sdesc(sa + TC_A_BYTES, 128, 256), sdesc(sb + N * 256, 128, 256), idesc, 0u);
      }
      mma_commit(empty + s);
    }
    mma_commit(accfull + b);
  }
done:
  mma_commit(drain);
  tc_drain(drain, 0);
}

// Final value of (global row, activation row b) through the epilogue operation
// (bias `brow` already loaded for the row). Every lane of the warp calls it with the
// same b (gated rows read their up row from lane + 8).
template <int EPI>
__device__ __forceinline__ void emit(const TcArgs &a, int row, int b, float v, float brow, int lane) {
  if constexpr (EPI == EPI_GLU_SILU || EPI == EPI_GLU_GELU) {
    const float u = __shfl_down_sync(0xffffffffu, v, 8);
    if ((lane & 8) == 0 && row < a.rows)
      a.y[(int64_t)b * a.ldy + (row >> 4) * 8 + (row & 7)] = (EPI == EPI_GLU_SILU ? tc_silu(v) : tc_gelu(v)) * u;
  } else {
    if (row >= a.rows) return;
    float *dst = a.y + (int64_t)b * a.ldy + row;
    if constexpr (EPI == EPI_ADD) *dst = __ldcg(dst) + (v + brow);  // residual read through L2
    else if constexpr (EPI == EPI_SILU) *dst = tc_silu(v + brow);
    else *dst = v + brow;
  }
}

// Y = Y + d*R - dmin*Mn for columns c..c+15 of this thread's row (Y absent on the
// first unit of a segment), then either kept in tensor memory or written out.
// (in place: r becomes the new Y, as float bits)
__device__ __forceinline__ void epi_cols16(uint32_t (&r)[16], const uint32_t (&mn)[16], const uint32_t (&yv)[16], bool first, float d,
                                           float dmin) {
#pragma unroll
  for (int j = 0; j < 16; j++)
    r[j] = __float_as_uint((first ? 0.f : __uint_as_float(yv[j])) + fmaf(d, __uint_as_float(r[j]), -dmin * __uint_as_float(mn[j])));
}

template <int EPI>
__device__ __forceinline__ void out_cols16(const TcArgs &a, const uint32_t (&v)[16], const float *cscale, int c, bool whole, int row,
                                           float brow, int lane, float *pdst) {
  float cs[16];
#pragma unroll
  for (int j = 0; j < 16; j += 4) {
    const float4 t = *reinterpret_cast<const float4 *>(cscale + c + j);
    cs[j] = t.x;
    cs[j + 1] = t.y;
    cs[j + 2] = t.z;
    cs[j + 3] = t.w;
  }
  if (whole) {
#pragma unroll
    for (int j = 0; j < 16; j++)
      if (c + j < a.batch) emit<EPI>(a, row, c + j, __uint_as_float(v[j]) * cs[j], brow, lane);
  } else {
#pragma unroll
    for (int j = 0; j < 16; j++)
      if (c + j < a.batch) pdst[(size_t)(c + j) * TC_M] = __uint_as_float(v[j]) * cs[j];
  }
}

template <int T, int EPI>
__device__ void role_epilogue(const TcArgs &a, uint32_t tbase, const float *cscale, uint64_t *accfull, uint64_t *accempty,
                              uint64_t *mnempty, volatile int *stop, int *pend, int u0, int u1, int q, int h, int lane) {
  const int N = a.N, m = 32 * q + lane;
  // this warp's 16-column chunks (h: which half of them when two warps share a lane quarter)
  const int nch = N / 16, half = TC_EPIW == 8 ? (nch + 1) / 2 : nch;
  const int cbeg = h ? 16 * half : 0, cend = h ? N : 16 * half;
  const uint32_t lt = tbase + ((uint32_t)(32 * q) << 16);
  const int cta = blockIdx.x;
  int i = 0;
  for (int U = u0; U < u1; U++, i++) {
    const UnitPos P = unit_pos(a, u0, u1, U);
    const int mt = P.mt, kb = P.kb, b = i & 1;
    const bool first = P.j == 0, last = P.j == P.len - 1, whole = P.len == a.nkb;
    const int row = mt * TC_M + m, tile = mt * TC_TILES + (m >> 4);
    // super-block scales of the row: Q4_K d | dmin (chunk bytes 2048 + 16r), Q6_K d (3328 + 2r)
    uint32_t hdr = 0;
    if (tile < a.tiles) {
      const uint8_t *ck = a.w + ((size_t)tile * a.nkb + kb) * TcType<T>::CHUNK;
      hdr = TcType<T>::MINS ? ldg_u32(ck + 2048 + 16 * (m & 15)) : ldg_u16(ck + 3328 + 2 * (m & 15));
    }
    float brow = 0.f;
    if (last && whole && a.bias && row < a.rows) brow = __ldg(a.bias + row);
    bool ok = tc_wait(accfull + b, (i >> 1) & 1, stop, a.status);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    const float d = h2f(hdr), dmin = TcType<T>::MINS ? h2f(hdr >> 16) : 0.f;
    const int slot = u0 >= mt * a.nkb ? 0 : 1;
    float *pdst = a.part + (size_t)(cta * 2 + slot) * N * TC_M + m;
    for (int c = cbeg; c < cend; c += 16) {
      uint32_t r0[16], m0[16], y0[16];
#pragma unroll
      for (int j = 0; j < 16; j++) r0[j] = m0[j] = y0[j] = 0u;
      if (ok) {
        tmem_ld16(lt + b * N + c, r0);
        if (TcType<T>::MINS) tmem_ld16(lt + 2 * N + c, m0);
        if (!first) tmem_ld16(lt + 3 * N + c, y0);
        tmem_wait_ld();
        reg_fence(r0);
        reg_fence(m0);
        reg_fence(y0);
      }
      epi_cols16(r0, m0, y0, first, d, dmin);
      if (!last) {
        if (ok) tmem_st16(lt + 3 * N + c, r0);
        continue;
      }
      out_cols16<EPI>(a, r0, cscale, c, whole, row, brow, lane, pdst);
    }
    if (!last && ok) tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(accempty + b);
      mbar_arrive(mnempty);
    }
    if (!last || whole) continue;
    // M-tile cut between CTAs: publish this CTA's partial (one arrival on the M-tile's
    // counter); the contributors sum the partials at the end of their ranges (finalize)
    __threadfence();
    epi_bar();
    if (q == 0 && h == 0 && lane == 0) {
      atomicAdd(a.ctr + mt, 1u);
      pend[slot] = mt;
    }
  }
}

// Output of 16 consecutive rows row0.. (one 16-row tile) of activation row b.
template <int EPI>
__device__ void emit16(const TcArgs &a, int row0, int b, const float (&v)[16]) {
  if constexpr (EPI == EPI_GLU_SILU || EPI == EPI_GLU_GELU) {
    float *dst = a.y + (int64_t)b * a.ldy + (row0 >> 4) * 8;
#pragma unroll
    for (int j = 0; j < 8; j++)
      if (row0 + j < a.rows) dst[j] = (EPI == EPI_GLU_SILU ? tc_silu(v[j]) : tc_gelu(v[j])) * v[j + 8];
  } else {
#pragma unroll
    for (int j = 0; j < 16; j++) {
      const int row = row0 + j;
      if (row >= a.rows) break;
      float x = v[j];
      if (a.bias) x += __ldg(a.bias + row);
      float *dst = a.y + (int64_t)b * a.ldy + row;
      if constexpr (EPI == EPI_ADD) *dst = __ldcg(dst) + x;
      else if constexpr (EPI == EPI_SILU) *dst = tc_silu(x);
      else *dst = x;
    }
  }
}

// M-tile mt was cut between CTAs c0..c1: once all of them have published their
// partials, CTA c0 + i sums (in CTA order) and writes activation rows
// [i*batch/C, (i+1)*batch/C) of it; the last to finish resets the counter.
// Whole CTA; every thread reaches both block barriers.
template <int EPI>
__device__ void finalize(const TcArgs &a, int mt, volatile int *stop) {
  const int c0 = unit_owner(a, mt * a.nkb), c1 = unit_owner(a, (mt + 1) * a.nkb - 1), C = c1 - c0 + 1;
  const int me = (int)blockIdx.x - c0;
  if (threadIdx.x == 0 && !*stop) {
    const uint64_t t0 = gtime();
    while (ld_acquire(a.ctr + mt) < (unsigned)C) {
      if (gtime() - t0 > TC_TIMEOUT_NS) {
        atomicCAS(a.status, 0, 1);
        *stop = 1;
        break;
      }
      __nanosleep(100);
    }
  }
  __syncthreads();
  if (!*stop) {
    const int b0 = me * a.batch / C, b1 = (me + 1) * a.batch / C, items = (b1 - b0) * TC_TILES;
    for (int it = threadIdx.x; it < items; it += blockDim.x) {
      const int b = b0 + it / TC_TILES, t = it % TC_TILES;
      float acc[16];
#pragma unroll
      for (int j = 0; j < 16; j++) acc[j] = 0.f;
      for (int cc = c0; cc <= c1; cc += 2) {
        float4 v[2][4];
#pragma unroll
        for (int g = 0; g < 2; g++) {
          if (cc + g > c1) break;
          const int sl = unit_start(a, cc + g) >= mt * a.nkb ? 0 : 1;
          const float4 *src = reinterpret_cast<const float4 *>(a.part + ((size_t)((cc + g) * 2 + sl) * a.N + b) * TC_M + 16 * t);
#pragma unroll
          for (int k = 0; k < 4; k++) v[g][k] = __ldcg(src + k);
        }
#pragma unroll
        for (int g = 0; g < 2; g++) {
          if (cc + g > c1) break;
#pragma unroll
          for (int k = 0; k < 4; k++) {
            acc[4 * k] += v[g][k].x;
            acc[4 * k + 1] += v[g][k].y;
            acc[4 * k + 2] += v[g][k].z;
            acc[4 * k + 3] += v[g][k].w;
          }
        }
      }
      emit16<EPI>(a, mt * TC_M + 16 * t, b, acc);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && !*stop) {
    const unsigned old = atomicAdd(a.ctr + mt, 1u);
    if (old == (unsigned)(2 * C - 1)) atomicExch(a.ctr + mt, 0u);
  }
}

template <int T, int EPI>
__global__ void __launch_bounds__(TC_THREADS, 1) gemm_tc_kernel(const TcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t *bfull = reinterpret_cast<uint64_t *>(smem), *afull = bfull + TC_MAXST, *empty = afull + TC_MAXST, *rawfull = empty + TC_MAXST,
           *rawempty = rawfull + 2, *accfull = rawempty + 2, *accempty = accfull + 2, *mnempty = accempty + 2,
           *drain = mnempty + 1;
  static_assert((3 * TC_MAXST + 10) * 8 <= 384, "barrier area");
  uint32_t *tslot = reinterpret_cast<uint32_t *>(smem + 384);
  volatile int *stop = reinterpret_cast<volatile int *>(smem + 388);
  int *pend = reinterpret_cast<int *>(smem + 392);  // M-tiles of this CTA's cut segments (first, last) or -1
  float *cscale = reinterpret_cast<float *>(smem + 512);  // N <= 128 floats
  uint8_t *raw = smem + TC_HDR;
  uint8_t *stages = raw + 2 * TC_TILES * TcType<T>::CHUNK;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, c = blockIdx.x;
  const int u0 = unit_start(a, c), u1 = unit_start(a, c + 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.nstage; s++) {
      mbar_init(bfull + s, 1);
      mbar_init(afull + s, TC_DQ);
      mbar_init(empty + s, 1);
    }
    for (int r = 0; r < 2; r++) {
      mbar_init(rawfull + r, 1);
      mbar_init(rawempty + r, TC_DQ);
      mbar_init(accfull + r, 1);
      mbar_init(accempty + r, TC_EPIW);
    }
    mbar_init(mnempty, TC_EPIW);
    mbar_init(drain, 1);
    *stop = 0;
    pend[0] = pend[1] = -1;
    fence_async_smem();
  }
  if (threadIdx.x < a.N)
    cscale[threadIdx.x] = reinterpret_cast<const float *>(a.panel + (size_t)a.nkb * panel_kb_bytes(a.N))[threadIdx.x];
  if (warp == TC_MMAW) {
    tmem_alloc(tslot, a.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;

  if (warp < TC_DQ) {
    role_dequant<T>(a, raw, stages, afull, empty, rawfull, rawempty, stop, u0, u1, warp, lane);
  } else if (warp < TC_EPI0 + TC_EPIW) {
    role_epilogue<T, EPI>(a, tbase, cscale, accfull, accempty, mnempty, stop, pend, u0, u1, warp & 3, 0, lane);
  } else if (warp == TC_RAWW) {
    if (lane == 0) role_raw<T>(a, raw, rawfull, rawempty, stop, u0, u1);
  } else if (warp == TC_BW) {
    if (lane == 0) role_b<T>(a, stages, bfull, empty, stop, u0, u1);
  } else if (warp == TC_MMAW) {
    if (lane == 0) role_mma<T>(a, tbase, stages, bfull, afull, empty, accfull, accempty, mnempty, drain, stop, u0, u1);
  }
  __syncwarp();  // single-lane roles reconverge before the block barrier
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == TC_MMAW) tmem_dealloc(tbase, a.tmem_cols);
  // cut M-tiles: the first segment's tile, then the last's (each CTA waits only for
  // contributors that publish before they finalize, so the waits cannot cycle)
  const int p0 = pend[0], p1 = pend[1];
  if (p0 >= 0) finalize<EPI>(a, p0, stop);
  if (p1 >= 0) finalize<EPI>(a, p1, stop);
}

// One block per activation row (N rows, rows >= batch are zero): optional
// RMSNorm, power-of-two row scale, f16 hi/lo split into the K-major core-matrix
// order of the B operand, and the hi/lo sub-block sums of the mins operand.
__global__ void __launch_bounds__(256) gemm_tc_prep_kernel(const float *x, int ldx, const float *norm_w, float eps, int batch,
                                                           int N, int cols, uint8_t *panel) {
  const int n = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ float red[8];
  __shared__ float s_inv, s_scale;
  const bool live = n < batch;
  const float *xr = x + (int64_t)n * ldx;
  float inv = 1.f;
  if (norm_w && live) {
    float s = 0.f;
    for (int c = tid; c < (cols >> 2); c += 256) {
      const float4 v = reinterpret_cast<const float4 *>(xr)[c];
      s = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, s))));
    }
    s = warp_sum(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (tid == 0) {
      float t = 0.f;
      for (int w = 0; w < 8; w++) t += red[w];
      s_inv = rsqrtf(t / (float)cols + eps);
    }
    __syncthreads();
    inv = s_inv;
  }
  float amax = 0.f;
  if (live) {
    for (int c = tid; c < (cols >> 2); c += 256) {
      float4 v = reinterpret_cast<const float4 *>(xr)[c];
      if (norm_w) {
        const float4 w = __ldg(reinterpret_cast<const float4 *>(norm_w) + c);
        v = make_float4(v.x * inv * w.x, v.y * inv * w.y, v.z * inv * w.z, v.w * inv * w.w);
      }
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
  }
  amax = warp_max(amax);
  __syncthreads();
  if (lane == 0) red[warp] = amax;
  __syncthreads();
  if (tid == 0) {
    float t = 0.f;
    for (int w = 0; w < 8; w++) t = fmaxf(t, red[w]);
    int e = 0;
    if (t > 0.f && isfinite(t)) {
      frexpf(t, &e);  // t = f * 2^e, f in [0.5, 1)
      e = min(max(10 - e, -120), 120);
    } else {
      e = 0;
    }
    s_scale = ldexpf(1.f, e);
    reinterpret_cast<float *>(panel + (size_t)(cols >> 8) * panel_kb_bytes(N))[n] = ldexpf(1.f, -e);
  }
  __syncthreads();
  const float sc = s_scale;
  const size_t kbb = panel_kb_bytes(N);
  for (int gi = tid; gi < (cols >> 3); gi += 256) {
    const int k = gi * 8, kb = k >> 8, k256 = k & 255, g = k256 >> 6, kk = k256 & 63;
    float v[8];
    if (live) {
      const float4 p0 = reinterpret_cast<const float4 *>(xr + k)[0], p1 = reinterpret_cast<const float4 *>(xr + k)[1];
      v[0] = p0.x; v[1] = p0.y; v[2] = p0.z; v[3] = p0.w; v[4] = p1.x; v[5] = p1.y; v[6] = p1.z; v[7] = p1.w;
      if (norm_w) {
        const float4 w0 = __ldg(reinterpret_cast<const float4 *>(norm_w + k)), w1 = __ldg(reinterpret_cast<const float4 *>(norm_w + k) + 1);
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = v[j] * inv * wv[j];
      }
#pragma unroll
      for (int j = 0; j < 8; j++) v[j] *= sc;
    } else {
#pragma unroll
      for (int j = 0; j < 8; j++) v[j] = 0.f;
    }
    uint32_t hi[4], lo[4];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const __half h0 = __float2half_rn(v[2 * j]), h1 = __float2half_rn(v[2 * j + 1]);
      hi[j] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
      lo[j] = h2pair(v[2 * j] - __half2float(h0), v[2 * j + 1] - __half2float(h1));
      s += v[2 * j] + v[2 * j + 1];
    }
    uint8_t *base = panel + (size_t)kb * kbb + (size_t)g * N * 256 + (n >> 3) * 1024 + (kk >> 3) * 128 + (n & 7) * 16;
    *reinterpret_cast<uint4 *>(base) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4 *>(base + (size_t)N * 128) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    // sub-block sums (32 columns = 4 consecutive threads)
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if ((gi & 3) == 0) {
      const int j = k256 >> 5;
      const __half sh = __float2half_rn(s);
      const __half sl = __float2half_rn(s - __half2float(sh));
      uint8_t *bm = panel + (size_t)kb * kbb + (size_t)4 * N * 256 + (n >> 3) * 256 + (n & 7) * 16 + j * 2;
      *reinterpret_cast<__half *>(bm) = sh;
      *reinterpret_cast<__half *>(bm + 128) = sl;
    }
  }
}

}  // namespace

bool gemm_tc_supported(int type, int rows, int cols, int batch) {
  return (type == Q4_K || type == Q6_K) && rows >= 1 && cols >= 256 && cols % 256 == 0 && batch >= 1 && batch <= GEMM_TC_MAX_BATCH;
}
size_t gemm_tc_panel_bytes(int batch, int cols) {
  const int N = (batch + 15) / 16 * 16;
  return (size_t)(cols / 256) * panel_kb_bytes(N) + (size_t)N * sizeof(float);
}
size_t gemm_tc_part_floats(int batch, int sm_count) {
  const int N = (batch + 15) / 16 * 16;
  return (size_t)sm_count * 2 * N * TC_M;
}
int gemm_tc_mtiles(int rows) { return (rows + TC_M - 1) / TC_M; }

cudaError_t launch_gemm_tc(const GemmTcLaunch &L, cudaStream_t s, int sm_count) {
  if (!gemm_tc_supported(L.type, L.rows, L.cols, L.batch) || sm_count < 1) return cudaErrorInvalidValue;
  const int N = (L.batch + 15) / 16 * 16;
  gemm_tc_prep_kernel<<<N, 256, 0, s>>>(L.x, L.ldx, L.norm_w, L.eps, L.batch, N, L.cols, L.panel);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  TcArgs a{};
  a.w = L.w;
  a.rows = L.rows;
  a.cols = L.cols;
  a.nkb = L.cols / 256;
  a.tiles = (L.rows + TILE_ROWS - 1) / TILE_ROWS;
  a.mtiles = gemm_tc_mtiles(L.rows);
  a.panel = L.panel;
  a.N = N;
  a.batch = L.batch;
  a.y = L.y;
  a.ldy = L.ldy;
  a.bias = L.bias;
  a.epi = L.epi;
  a.part = L.part;
  a.ctr = L.ctr;
  a.status = L.status;
  a.sbytes = stage_bytes(L.type, N);
  a.nstage = (int)((TC_SMEM_MAX - TC_HDR - 2 * raw_bytes(L.type)) / a.sbytes);
  if (a.nstage > TC_MAXST) a.nstage = TC_MAXST;
  if (a.nstage < 2) return cudaErrorInvalidValue;
  uint32_t cols = 32;
  while (cols < (uint32_t)(4 * N)) cols <<= 1;
  a.tmem_cols = cols;
  const int units = a.mtiles * a.nkb;
  const int grid = units < sm_count ? units : sm_count;
  a.q = units / grid;
  a.rem = units % grid;
  a.thr = a.rem * (a.q + 1);
  const size_t smem = (size_t)TC_HDR + 2 * raw_bytes(L.type) + (size_t)a.nstage * a.sbytes;
  if (L.epi < 0 || L.epi > EPI_GLU_GELU) return cudaErrorInvalidValue;
  using Kern = void (*)(const TcArgs);
  static const Kern table[2][5] = {
      {gemm_tc_kernel<Q4_K, EPI_STORE>, gemm_tc_kernel<Q4_K, EPI_ADD>, gemm_tc_kernel<Q4_K, EPI_SILU>,
       gemm_tc_kernel<Q4_K, EPI_GLU_SILU>, gemm_tc_kernel<Q4_K, EPI_GLU_GELU>},
      {gemm_tc_kernel<Q6_K, EPI_STORE>, gemm_tc_kernel<Q6_K, EPI_ADD>, gemm_tc_kernel<Q6_K, EPI_SILU>,
       gemm_tc_kernel<Q6_K, EPI_GLU_SILU>, gemm_tc_kernel<Q6_K, EPI_GLU_GELU>}};
  const int ti = L.type == Q4_K ? 0 : 1;
  const Kern kern = table[ti][L.epi];
  static bool attr[2][5] = {};
  if (!attr[ti][L.epi]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM_MAX);
    if (e != cudaSuccess) return e;
    cudaFuncAttributes fa;
    if ((e = cudaFuncGetAttributes(&fa, kern)) != cudaSuccess) return e;
    if (fa.maxThreadsPerBlock < TC_THREADS) return cudaErrorLaunchOutOfResources;  // register budget of the build
    attr[ti][L.epi] = true;
  }
  kern<<<grid, TC_THREADS, smem, s>>>(a);
  return cudaGetLastError();
}

}  // namespace wgd
