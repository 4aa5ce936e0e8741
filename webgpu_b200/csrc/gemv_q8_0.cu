// GEMV instantiations for Q8_0 weights (see gemv_impl.cuh).
#include "gemv_impl.cuh"
namespace wgd {
cudaError_t launch_gemv_q8_0(const GemvArgs &a, cudaStream_t s, bool pdl, int sm_count) {
  return launch_gemv_type<Q8_0>(a, s, pdl, sm_count);
}
}  // namespace wgd
