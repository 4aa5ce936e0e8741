// GEMV instantiations for Q5_K weights (see gemv_impl.cuh).
#include "gemv_impl.cuh"
namespace wgd {
cudaError_t launch_gemv_q5_k(const GemvArgs &a, cudaStream_t s, bool pdl, int sm_count) {
  return launch_gemv_type<Q5_K>(a, s, pdl, sm_count);
}
}  // namespace wgd
