// GEMV instantiations per GGML type (row layout, gemv_impl.cuh), one launcher each for the
// dispatch in gemv.cu.
#include "gemv_impl.cuh"
namespace wgd {
cudaError_t launch_gemv_f32(const GemvArgs &a, cudaStream_t s, bool pdl, int sm_count) { return launch_gemv_type<F32>(a, s, pdl, sm_count); }
cudaError_t launch_gemv_f16(const GemvArgs &a, cudaStream_t s, bool pdl, int sm_count) { return launch_gemv_type<F16>(a, s, pdl, sm_count); }
cudaError_t launch_gemv_q4_0(const GemvArgs &a, cudaStream_t s, bool pdl, int sm_count) { return launch_gemv_type<Q4_0>(a, s, pdl, sm_count); }
cudaError_t launch_gemv_q8_0(const GemvArgs &a, cudaStream_t s, bool pdl, int sm_count) { return launch_gemv_type<Q8_0>(a, s, pdl, sm_count); }
cudaError_t launch_gemv_q4_k(const GemvArgs &a, cudaStream_t s, bool pdl, int sm_count) { return launch_gemv_type<Q4_K>(a, s, pdl, sm_count); }
cudaError_t launch_gemv_q5_k(const GemvArgs &a, cudaStream_t s, bool pdl, int sm_count) { return launch_gemv_type<Q5_K>(a, s, pdl, sm_count); }
cudaError_t launch_gemv_q6_k(const GemvArgs &a, cudaStream_t s, bool pdl, int sm_count) { return launch_gemv_type<Q6_K>(a, s, pdl, sm_count); }
}  // namespace wgd
