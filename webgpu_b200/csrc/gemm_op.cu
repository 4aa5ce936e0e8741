// wgd_op_gemm_tiled / wgd_op_gemm_tiled_status: the prompt-batch tcgen05 GEMM
// (gemm_tc.cu) as a standalone C-ABI operation, with per-device scratch (the
// prepared activation panel, split-K partials, M-tile counters and the status
// word) grown on demand. Calls on one device share the scratch, so they must be
// ordered (one stream, or the caller serialises them).
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "kernels.h"
#include "tile.cuh"
#include "wgd.h"

namespace wgd {
int api_fail(int code, const std::string &msg);
}

namespace {
using namespace wgd;

constexpr int kMaxDevices = 16;

struct GemmScratch {
  uint8_t *panel = nullptr;
  size_t panel_n = 0;
  float *part = nullptr;
  size_t part_n = 0;
  unsigned *ctr = nullptr;
  int ctr_n = 0;
  int *status = nullptr;
  int sm = 0;
};
std::mutex g_mu;
GemmScratch g_s[kMaxDevices];

#define CKG(x)                                                                          \
  do {                                                                                  \
    cudaError_t e_ = (x);                                                               \
    if (e_ != cudaSuccess) return api_fail(WGD_ECUDA, std::string(#x) + ": " + cudaGetErrorString(e_)); \
  } while (0)

}  // namespace

extern "C" int wgd_op_gemm_tiled(int type, int64_t rows, int64_t cols, const void *tiled, const float *x, int batch, float *y,
                                 void *stream) {
  if (!tiled || !x || !y) return api_fail(WGD_EINVAL, "null argument");
  if (rows < 1 || rows > (1 << 24) || cols < 256 || cols > (1 << 20) ||
      !gemm_tc_supported(type, (int)rows, (int)cols, batch))
    return api_fail(WGD_EINVAL, "the tensor-core GEMM takes Q4_K or Q6_K, whole super-blocks and 1..128 activation rows");
  int dev = 0;
  CKG(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return api_fail(WGD_EINVAL, "device index");
  GemmScratch *S = &g_s[dev];
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!S->status) {
      cudaDeviceProp p;
      CKG(cudaGetDeviceProperties(&p, dev));
      S->sm = p.multiProcessorCount;
      CKG(cudaMalloc(&S->status, sizeof(int)));
      CKG(cudaMemset(S->status, 0, sizeof(int)));
    }
    const size_t pb = gemm_tc_panel_bytes(batch, (int)cols), pf = gemm_tc_part_floats(batch, S->sm);
    const int mt = gemm_tc_mtiles((int)rows);
    if (S->panel_n < pb) {
      if (S->panel) cudaFree(S->panel);
      S->panel = nullptr;
      CKG(cudaMalloc(&S->panel, pb));
      S->panel_n = pb;
    }
    if (S->part_n < pf) {
      if (S->part) cudaFree(S->part);
      S->part = nullptr;
      CKG(cudaMalloc(&S->part, pf * sizeof(float)));
      S->part_n = pf;
    }
    if (S->ctr_n < mt) {
      if (S->ctr) cudaFree(S->ctr);
      S->ctr = nullptr;
      CKG(cudaMalloc(&S->ctr, mt * sizeof(unsigned)));
      CKG(cudaMemset(S->ctr, 0, mt * sizeof(unsigned)));
      S->ctr_n = mt;
    }
  }
  GemmTcLaunch g{};
  g.type = type;
  g.w = (const uint8_t *)tiled;
  g.rows = (int)rows;
  g.cols = (int)cols;
  g.x = x;
  g.ldx = (int)cols;
  g.eps = 0.f;
  g.y = y;
  g.ldy = (int)rows;
  g.epi = EPI_STORE;
  g.batch = batch;
  g.panel = S->panel;
  g.part = S->part;
  g.ctr = S->ctr;
  g.status = S->status;
  CKG(launch_gemm_tc(g, (cudaStream_t)stream, S->sm));
  return WGD_OK;
}

extern "C" int wgd_op_gemm_tiled_status(int *status) {
  if (!status) return api_fail(WGD_EINVAL, "null argument");
  int dev = 0;
  CKG(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return api_fail(WGD_EINVAL, "device index");
  *status = 0;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_s[dev].status) return WGD_OK;
  CKG(cudaDeviceSynchronize());
  CKG(cudaMemcpy(status, g_s[dev].status, sizeof(int), cudaMemcpyDeviceToHost));
  CKG(cudaMemset(g_s[dev].status, 0, sizeof(int)));
  return WGD_OK;
}
