// GEMV instantiations for F32 weights (see gemv_impl.cuh).
#include "gemv_impl.cuh"
namespace wgd {
cudaError_t launch_gemv_f32(const GemvArgs &a, cudaStream_t s, bool pdl, int sm_count) {
  return launch_gemv_type<F32>(a, s, pdl, sm_count);
}
}  // namespace wgd
