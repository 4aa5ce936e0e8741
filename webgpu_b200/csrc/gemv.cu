// GEMV dispatch by GGML type; batches wider than one register pass are split.
#include "kernels.h"
#include "common.cuh"

namespace wgd {
cudaError_t launch_gemv_f32(const GemvArgs &, cudaStream_t, bool, int);
cudaError_t launch_gemv_f16(const GemvArgs &, cudaStream_t, bool, int);
cudaError_t launch_gemv_q4_0(const GemvArgs &, cudaStream_t, bool, int);
cudaError_t launch_gemv_q8_0(const GemvArgs &, cudaStream_t, bool, int);
cudaError_t launch_gemv_q4_k(const GemvArgs &, cudaStream_t, bool, int);
cudaError_t launch_gemv_q5_k(const GemvArgs &, cudaStream_t, bool, int);
cudaError_t launch_gemv_q6_k(const GemvArgs &, cudaStream_t, bool, int);

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
