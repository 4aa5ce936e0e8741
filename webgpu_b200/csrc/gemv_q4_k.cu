// GEMV instantiations for Q4_K weights (see gemv_impl.cuh).
#include "gemv_impl.cuh"
namespace wgd {
cudaError_t launch_gemv_q4_k(const GemvArgs &a, cudaStream_t s, bool pdl, int sm_count) {
  return launch_gemv_type<Q4_K>(a, s, pdl, sm_count);
}
}  // namespace wgd
