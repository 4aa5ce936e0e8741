// GEMV instantiations for F16 weights (see gemv_impl.cuh).
#include "gemv_impl.cuh"
namespace wgd {
cudaError_t launch_gemv_f16(const GemvArgs &a, cudaStream_t s, bool pdl, int sm_count) {
  return launch_gemv_type<F16>(a, s, pdl, sm_count);
}
}  // namespace wgd
