// Tile-16 weight layout for the tensor-core GEMV (gemv2_impl.cuh).
//
// Rows are grouped in tiles of 16 (the M of an mma.sync m16n8k32/k16 tile;
// the last tile is zero-padded). A tile row is a sequence of K-chunks of one
// GGUF block column (256 values for K-quants), each chunk holding that block
// of all 16 rows: 16 x block_bytes bytes, the same bytes as GGUF, reordered so
// that every lane of a warp fetches exactly the integers of its MMA fragment
// with coalesced 16-byte loads:
//
//  Q4_K chunk (2304 B)
//    [0, 2048)     qs: for sub-block pair g (sub-blocks 2g low nibbles, 2g+1
//                  high nibbles) 512 B; lane l = 4*grp + tig owns 16 B:
//                  words {row grp, row grp+8} x {qs bytes 32g+4tig.., 32g+16+4tig..}
//                  ordered (row grp, lo16), (row grp+8, lo16), (row grp, hi16), (row grp+8, hi16)
//                  = the A fragment a0..a3 of m16n8k32 before nibble unpacking.
//    [2048, 2304)  16 rows x 16 B: d, dmin, 12 scale/min bytes (GGUF order).
//  Q6_K chunk (3360 B)
//    [0, 2048)     ql: 4 regions k = 2*seg + qp of 512 B; lane l owns 16 B:
//                  words (row grp, h0), (row grp+8, h0), (row grp, h1), (row grp+8, h1)
//                  = ql bytes seg*64 + qp*32 + 16h + 4tig .. +3 of that row.
//    [2048, 3072)  qh: 2 regions seg of 512 B, same word order over
//                  qh bytes seg*32 + 16h + 4tig .. +3.
//    [3072, 3328)  16 rows x 16 int8 scales.
//    [3328, 3360)  16 rows x fp16 d.
#pragma once
#include "common.cuh"

namespace wgd {

constexpr int TILE_ROWS = 16;

inline bool tiled_type(int t) { return t == Q4_K || t == Q6_K; }
inline int64_t tile_chunk_bytes(int t) { return 16LL * block_bytes(t); }
inline int64_t tiled_bytes(int t, int64_t rows, int64_t cols) {
  return (rows + 15) / 16 * (cols / block_elems(t)) * tile_chunk_bytes(t);
}

// Destination offset (inside a chunk) of raw byte `b` of the GGUF block of local row r.
__host__ __device__ inline int tile_offset(int type, int r, int b) {
  const int grp = r & 7, rowsel = r >> 3;
  if (type == Q4_K) {
    if (b < 16) return 2048 + 16 * r + b;
    const int qb = b - 16, g = qb >> 5, k = qb & 31;
    const int tig = (k & 15) >> 2, part = k >> 4, byte = k & 3;
    return 512 * g + 16 * (grp * 4 + tig) + 4 * (part * 2 + rowsel) + byte;
  }
  // Q6_K
  if (b < 128) {
    const int seg = b >> 6, qp = (b & 63) >> 5, l = b & 31;
    const int h = l >> 4, tig = (l & 15) >> 2, byte = l & 3;
    return (2 * seg + qp) * 512 + 16 * (grp * 4 + tig) + 4 * (h * 2 + rowsel) + byte;
  }
  if (b < 192) {
    const int hb = b - 128, seg = hb >> 5, l = hb & 31;
    const int h = l >> 4, tig = (l & 15) >> 2, byte = l & 3;
    return 2048 + seg * 512 + 16 * (grp * 4 + tig) + 4 * (h * 2 + rowsel) + byte;
  }
  if (b < 208) return 3072 + 16 * r + (b - 192);
  return 3328 + 2 * r + (b - 208);
}

// Bit-exact dequant of (row, col) from the tiled layout (WGSL f32 order, as
// dequant_elem in quant.cuh).
template <int T>
__device__ __forceinline__ float dequant_tiled(const uint8_t *w, int nkb, int row, int col) {
  constexpr int BB = T == Q4_K ? 144 : 210;
  const int t = row >> 4, r = row & 15, kb = col >> 8, j = col & 255;
  const uint8_t *c = w + ((int64_t)t * nkb + kb) * (16 * BB);
  if (T == Q4_K) {
    const int s = j >> 5;
    const uint8_t *h = c + 2048 + 16 * r;
    const float d = h2f((uint32_t)h[0] | ((uint32_t)h[1] << 8)), dmin = h2f((uint32_t)h[2] | ((uint32_t)h[3] << 8));
    const uint8_t *S = h + 4;
    uint32_t sc, mn;
    if (s < 4) { sc = S[s] & 63u; mn = S[4 + s] & 63u; }
    else { sc = (S[4 + s] & 15u) | ((S[s - 4] >> 6u) << 4u); mn = (S[4 + s] >> 4u) | ((S[s] >> 6u) << 4u); }
    const int qb = 16 + (j >> 6) * 32 + (j & 31);
    const uint32_t q = (c[tile_offset(Q4_K, r, qb)] >> ((s & 1) * 4)) & 15u;
    return __fsub_rn(__fmul_rn(d, (float)(sc * q)), __fmul_rn(dmin, (float)mn));
  } else {
    const int segment = j >> 7, quarter = (j & 127) >> 5, lane = j & 31;
    const uint32_t low = (c[tile_offset(Q6_K, r, segment * 64 + (quarter & 1) * 32 + lane)] >> ((quarter >> 1) * 4)) & 15u;
    const uint32_t high = (c[tile_offset(Q6_K, r, 128 + segment * 32 + lane)] >> (quarter * 2)) & 3u;
    const int sc = (int8_t)c[3072 + 16 * r + segment * 8 + quarter * 2 + (lane >> 4)];
    const float d = h2f((uint32_t)c[3328 + 2 * r] | ((uint32_t)c[3329 + 2 * r] << 8));
    return __fmul_rn(__fmul_rn(d, (float)sc), (float)((int)(low | (high << 4)) - 32));
  }
}

}  // namespace wgd
