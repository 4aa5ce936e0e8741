// Tensor-core GEMV instantiations for Q4_K tiles (see gemv2_impl.cuh).
#include "gemv2_impl.cuh"
namespace wgd {
cudaError_t launch_gemv2_q4_k(const Gemv2Args &a, cudaStream_t s, bool pdl, int sm_count) {
  return launch_gemv2_type<Q4_K>(a, s, pdl, sm_count);
}
}  // namespace wgd
