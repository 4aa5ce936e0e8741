// wgd_op_gemv_tiled_noalloc: the tiled tensor-core GEMV of wgd_op_gemv_tiled with
// its scratch (stream-K partial sums and split-tile counters) in one fixed
// file-scope device array instead of cudaMalloc'd memory, for callers that may
// not allocate device memory once they are running.
//
// The first call on each device (with that device current) looks the array up
// with cudaGetSymbolAddress and reads the SM count; that first call should come
// before any stream capture, and it is the only one that may make the CUDA
// runtime load the module. Every call allocates nothing. The split-tile
// counters need no clearing: the array is zero-initialised when the module
// loads on a device, and every call leaves the counters at zero again. The
// cached address assumes the CUDA context of the device lives as long as the
// process (after a cudaDeviceReset it would be stale). The array is one per
// device, so calls on the same device must not overlap in time (two streams
// running this entry point concurrently share the partials and counters and
// race).
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

// 4 MiB of partial sums covers every projection of a 4096-wide model up to
// 4096 x 14336 and 65536 x 4096; 8192 counters cover 131072 rows.
constexpr size_t kPartFloats = size_t(1) << 20;
constexpr int kTileCounters = 8192;
constexpr size_t kPartBytes = kPartFloats * sizeof(float);
constexpr size_t kScratchBytes = kPartBytes + kTileCounters * sizeof(unsigned);
constexpr int kMaxDevices = 16;

struct DeviceScratch {
  bool ready = false;
  float *part = nullptr;
  unsigned *ctr = nullptr;
  int sm = 0;
};
DeviceScratch g_dev[kMaxDevices];
std::mutex g_mu;

int cuda_fail(const char *what, cudaError_t e) { return api_fail(WGD_ECUDA, std::string(what) + ": " + cudaGetErrorString(e)); }
}  // namespace

static __device__ __align__(256) unsigned char g_gemv_scratch[kScratchBytes];

extern "C" int wgd_op_gemv_tiled_noalloc(int type, int64_t rows, int64_t cols, const void *tiled, const float *x, int batch,
                                         float *y, void *stream) {
  if (!tiled_type(type) || cols % 256 || rows < 1 || rows > (1 << 30) || batch < 1 || gemv2_max_batch((int)cols) == 0)
    return api_fail(WGD_EINVAL, "bad type, shape or batch for the tiled GEMV");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail("cudaGetDevice", e);
  if (dev < 0 || dev >= kMaxDevices) return api_fail(WGD_EINVAL, "device index");
  DeviceScratch s;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceScratch &d = g_dev[dev];
    if (!d.ready) {  // setup, once per device
      void *base = nullptr;
      if ((e = cudaGetSymbolAddress(&base, g_gemv_scratch)) != cudaSuccess) return cuda_fail("cudaGetSymbolAddress(gemv scratch)", e);
      int sm = 0;
      if ((e = cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
        return cuda_fail("cudaDeviceGetAttribute(SM count)", e);
      unsigned char *b = static_cast<unsigned char *>(base);
      d.part = reinterpret_cast<float *>(b);
      d.ctr = reinterpret_cast<unsigned *>(b + kPartBytes);
      d.sm = sm;
      d.ready = true;
    }
    s = d;
  }
  const size_t need = gemv2_part_floats(type, (int)rows, (int)cols, s.sm);
  const int64_t tiles = (rows + 15) / 16;
  if (need > kPartFloats || tiles > kTileCounters)
    return api_fail(WGD_EINVAL, "tiled GEMV " + std::to_string(rows) + "x" + std::to_string(cols) + " needs " +
                                    std::to_string(need) + " partial floats and " + std::to_string(tiles) +
                                    " tile counters; the fixed scratch holds " + std::to_string(kPartFloats) + " and " +
                                    std::to_string(kTileCounters) + " (wgd_op_gemv_tiled has no such limit)");
  Gemv2Launch g{};
  g.w = static_cast<const uint8_t *>(tiled);
  g.rows = (int)rows;
  g.cols = (int)cols;
  g.x = x;
  g.ldx = (int)cols;
  g.eps = 0.f;
  g.y = y;
  g.ldy = (int)rows;
  g.epi = EPI_STORE;
  g.batch = batch;
  g.part = s.part;
  g.part_floats = kPartFloats;
  g.tile_ctr = s.ctr;
  g.ctr_count = kTileCounters;
  if ((e = launch_gemv2(type, g, (cudaStream_t)stream, false, s.sm)) != cudaSuccess) return cuda_fail("tiled GEMV launch", e);
  return WGD_OK;
}
