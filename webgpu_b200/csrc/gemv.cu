// GEMV dispatch by GGML type; batches wider than one register pass are split.
#include "kernels.h"
#include "common.cuh"
#include "gemv2_impl.cuh"

namespace wgd {
// row-layout instantiations: gemv_types.cu
cudaError_t launch_gemv_f32(const GemvArgs &, cudaStream_t, bool, int);
cudaError_t launch_gemv_f16(const GemvArgs &, cudaStream_t, bool, int);
cudaError_t launch_gemv_q4_0(const GemvArgs &, cudaStream_t, bool, int);
cudaError_t launch_gemv_q8_0(const GemvArgs &, cudaStream_t, bool, int);
cudaError_t launch_gemv_q4_k(const GemvArgs &, cudaStream_t, bool, int);
cudaError_t launch_gemv_q5_k(const GemvArgs &, cudaStream_t, bool, int);
cudaError_t launch_gemv_q6_k(const GemvArgs &, cudaStream_t, bool, int);
// tensor-core GEMV instantiations for the tiled Q4_K / Q6_K layout (gemv2_impl.cuh)
cudaError_t launch_gemv2_q4_k(const Gemv2Args &a, cudaStream_t s, bool pdl, int sm_count) {
  return launch_gemv2_type<Q4_K>(a, s, pdl, sm_count);
}
cudaError_t launch_gemv2_q6_k(const Gemv2Args &a, cudaStream_t s, bool pdl, int sm_count) {
  return launch_gemv2_type<Q6_K>(a, s, pdl, sm_count);
}

int gemv_max_batch(int cols) {
  if (cols % 32) return 0;
  if (cols <= 8192) return 4;
  if (cols <= 16384) return 2;
  if (cols <= 24576) return 1;
  return 0;
}

static cudaError_t one(int type, const GemvArgs &a, cudaStream_t s, bool pdl, int sm) {
  switch (type) {
    case F32: return launch_gemv_f32(a, s, pdl, sm);
    case F16: return launch_gemv_f16(a, s, pdl, sm);
    case Q4_0: return launch_gemv_q4_0(a, s, pdl, sm);
    case Q8_0: return launch_gemv_q8_0(a, s, pdl, sm);
    case Q4_K: return launch_gemv_q4_k(a, s, pdl, sm);
    case Q5_K: return launch_gemv_q5_k(a, s, pdl, sm);
    case Q6_K: return launch_gemv_q6_k(a, s, pdl, sm);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_gemv(int type, const GemvArgs &a, cudaStream_t s, bool pdl, int sm_count) {
  const int chunk = gemv_max_batch(a.cols);
  if (chunk == 0 || a.batch < 1 || a.rows < 1) return cudaErrorInvalidValue;
  for (int b0 = 0; b0 < a.batch; b0 += chunk) {
    GemvArgs c = a;
    c.batch = a.batch - b0 < chunk ? a.batch - b0 : chunk;
    c.x = a.x + (int64_t)b0 * a.ldx;
    c.y = a.y + (int64_t)b0 * a.ldy;
    cudaError_t e = one(type, c, s, pdl && b0 == 0, sm_count);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}
}  // namespace wgd

namespace wgd {
int gemv2_max_batch(int cols) {
  if (cols % 256) return 0;
  if (cols <= 8192) return 4;
  if (cols <= 16384) return 2;
  if (cols <= 32768) return 1;
  return 0;
}

size_t gemv2_part_floats(int type, int rows, int cols, int sm_count) {
  (void)type;
  const int tiles = (rows + 15) / 16, nkb = cols / 256;
  // upper bound on the workers (8 CTAs of G2_WARPS warps per SM): fewer workers never touch a tile more often
  const int maxc = gemv2_maxc(tiles, nkb, (long long)sm_count * 8 * G2_WARPS);
  return (size_t)tiles * maxc * 16 * 4;
}

cudaError_t launch_gemv2(int type, const Gemv2Launch &l, cudaStream_t s, bool pdl, int sm_count) {
  const int chunk = gemv2_max_batch(l.cols);
  if (chunk == 0 || l.batch < 1 || l.rows < 1) return cudaErrorInvalidValue;
  Gemv2Args a{};
  a.w = l.w;
  a.rows = l.rows;
  a.cols = l.cols;
  a.tiles = (l.rows + 15) / 16;
  a.nkb = l.cols / 256;
  a.ldx = l.ldx;
  a.norm_w = l.norm_w;
  a.eps = l.eps;
  a.ldy = l.ldy;
  a.bias = l.bias;
  a.epi = l.epi;
  a.tile_ctr = l.tile_ctr;
  a.part = l.part;
  a.maxc = gemv2_maxc(a.tiles, a.nkb, (long long)sm_count * 8 * G2_WARPS);
  if (a.tiles > l.ctr_count || (size_t)a.tiles * a.maxc * 16 * 4 > l.part_floats) return cudaErrorInvalidValue;
  for (int b0 = 0; b0 < l.batch; b0 += chunk) {
    a.batch = l.batch - b0 < chunk ? l.batch - b0 : chunk;
    a.x = l.x + (int64_t)b0 * l.ldx;
    a.y = l.y + (int64_t)b0 * l.ldy;
    cudaError_t e = type == Q4_K ? launch_gemv2_q4_k(a, s, pdl && b0 == 0, sm_count)
                  : type == Q6_K ? launch_gemv2_q6_k(a, s, pdl && b0 == 0, sm_count) : cudaErrorInvalidValue;
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}
}  // namespace wgd
