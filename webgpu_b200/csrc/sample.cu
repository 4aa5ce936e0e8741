// Temperature / top-k / top-p sampling on the device over one row of logits: the
// reference's sample() (src/core/engine.ts:305-324) without the full-vocabulary
// readback.
//
// Candidate order. The reference keeps a list sorted by value with a stable sort, so
// among equal values the lower index comes first, and a value equal to the list's
// last entry does not enter a full list: the list is the top_k finite logits by
// (value descending, index ascending). Here each finite logit becomes one 64-bit key,
// (order-preserving bits of the value) << 32 | (0xffffffff - index), with -0 read as
// +0 (equal values in the reference), and non-finite logits key 0; keys are unique
// and a larger key is an earlier candidate.
//
// One launch: every CTA sorts its contiguous share of the row in shared memory
// (bitonic, 2048 keys a pass, the best 256 carried between passes) and publishes its
// top_k keys; the last CTA to finish keeps only keys at or above the largest of the
// CTAs' k-th keys (no global top-k candidate lies below it), sorts those the same way,
// and draws. The draw repeats the reference's double arithmetic in its order:
// p = exp((v - best) / temperature), total and the nucleus mass summed in candidate
// order, draw = uniform * retained, subtracted in order, falling back to the best.
// Every double operation is an explicit round-to-nearest intrinsic, so no step is
// contracted; exp() is CUDA's double exp, so a token can differ from a host draw only
// when the draw lies within a few ulp of a boundary between two candidates.
#include <cstdint>
#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels.h"
#include "wgd.h"

namespace wgd {
namespace {

constexpr int SMP_THREADS = 512;
constexpr int SMP_BUF = 2048;   // keys per sort pass
constexpr int SMP_KEEP = 256;   // best keys carried between passes (>= SAMPLE_MAX_K)
constexpr int SMP_MIN_SHARE = 1024;
static_assert(SMP_KEEP >= SAMPLE_MAX_K, "carried keys must cover top_k");

__device__ __forceinline__ uint64_t smp_key(float v, int64_t i) {
  if (!isfinite(v)) return 0ull;
  uint32_t b = v == 0.f ? 0u : __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((uint64_t)b << 32) | (uint64_t)(0xffffffffu - (uint32_t)i);
}
__device__ __forceinline__ float smp_value(uint64_t k) {
  uint32_t b = (uint32_t)(k >> 32);
  b = (b & 0x80000000u) ? (b & 0x7fffffffu) : ~b;
  return __uint_as_float(b);
}
__device__ __forceinline__ int smp_index(uint64_t k) { return (int)(0xffffffffu - (uint32_t)k); }

// Sorts s[0, SMP_BUF) descending (bitonic network; all threads of the CTA).
__device__ void smp_sort(uint64_t *s) {
  for (int k = 2; k <= SMP_BUF; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < SMP_BUF / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (j - 1)), hi = lo + j;
        const uint64_t a = s[lo], b = s[hi];
        const bool desc = (lo & k) == 0;
        if (desc ? a < b : a > b) {
          s[lo] = b;
          s[hi] = a;
        }
      }
      __syncthreads();
    }
}

// Leaves the SMP_KEEP largest of the keys get(0..count) in s[0, SMP_KEEP), descending
// (zeros where there are fewer).
template <class Get>
__device__ void smp_top(uint64_t *s, int64_t count, Get get) {
  for (int i = threadIdx.x; i < SMP_BUF; i += blockDim.x) s[i] = i < count ? get(i) : 0ull;
  __syncthreads();
  smp_sort(s);
  for (int64_t off = SMP_BUF; off < count; off += SMP_BUF - SMP_KEEP) {
    for (int i = threadIdx.x; i < SMP_BUF - SMP_KEEP; i += blockDim.x) s[SMP_KEEP + i] = off + i < count ? get(off + i) : 0ull;
    __syncthreads();
    smp_sort(s);
  }
}

__global__ void __launch_bounds__(SMP_THREADS) sample_kernel(SampleArgs a) {
  __shared__ uint64_t s[SMP_BUF];
  __shared__ double prob[SAMPLE_MAX_K];
  __shared__ int off[SAMPLE_MAX_GRID + 1];
  __shared__ uint64_t thr_s;
  __shared__ int last_s;
  pdl_wait();
  const SampleParams P = *a.params;
  const int K = P.top_k, G = gridDim.x, c = blockIdx.x;
  const int64_t lo = (int64_t)a.n * c / G, hi = (int64_t)a.n * (c + 1) / G;
  smp_top(s, hi - lo, [&](int64_t i) { return smp_key(__ldcg(a.logits + lo + i), lo + i); });
  for (int i = threadIdx.x; i < K; i += blockDim.x) a.part[(int64_t)c * K + i] = s[i];
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last_s = atomicAdd(a.ctr, 1u) == (unsigned)G - 1;
  __syncthreads();
  if (!last_s) return;
  __threadfence();

  // threshold: the largest k-th key of the CTAs (at least key 1: no non-finite logit)
  if (threadIdx.x == 0) thr_s = 1ull;
  __syncthreads();
  for (int l = threadIdx.x; l < G; l += blockDim.x) atomicMax((unsigned long long *)&thr_s, (unsigned long long)__ldcg(a.part + (int64_t)l * K + K - 1));
  __syncthreads();
  const uint64_t thr = thr_s;
  // keys >= thr of each (descending) list: a binary search for the first one below
  for (int l = threadIdx.x; l < G; l += blockDim.x) {
    const uint64_t *L = a.part + (int64_t)l * K;
    int lo2 = 0, hi2 = K;
    while (lo2 < hi2) {
      const int mid = (lo2 + hi2) >> 1;
      if (__ldcg(L + mid) >= thr) lo2 = mid + 1;
      else hi2 = mid;
    }
    off[l + 1] = lo2;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    off[0] = 0;
    for (int l = 0; l < G; l++) off[l + 1] += off[l];
  }
  __syncthreads();
  smp_top(s, off[G], [&](int64_t i) {
    int l0 = 0, l1 = G;  // list l with off[l] <= i < off[l + 1]
    while (l1 - l0 > 1) {
      const int m = (l0 + l1) >> 1;
      if (off[m] <= i) l0 = m;
      else l1 = m;
    }
    return __ldcg(a.part + (int64_t)l0 * K + (i - off[l0]));
  });

  // the draw
  const uint64_t top = s[0];
  const double best = (double)smp_value(top);
  if (P.temperature != 0.0)
    for (int j = threadIdx.x; j < K; j += blockDim.x)
      prob[j] = s[j] ? exp(__ddiv_rn(__dsub_rn((double)smp_value(s[j]), best), P.temperature)) : 0.0;
  __syncthreads();
  if (threadIdx.x == 0) {
    int token;
    if (!top) {
      token = -1;
    } else if (P.temperature == 0.0) {
      token = smp_index(top);
    } else {
      int count = 0;
      while (count < K && s[count]) count++;
      double total = 0.0;
      for (int j = 0; j < count; j++) total = __dadd_rn(total, prob[j]);
      double retained = 0.0;
      int cutoff = 0;
      for (; cutoff < count; cutoff++) {
        retained = __dadd_rn(retained, prob[cutoff]);
        if (__ddiv_rn(retained, total) >= P.top_p) {
          cutoff++;
          break;
        }
      }
      const double u = a.uniform[a.step ? __ldcg(a.step) : 0];
      double draw = __dmul_rn(u, retained);
      token = smp_index(top);
      for (int j = 0; j < cutoff; j++) {
        draw = __dsub_rn(draw, prob[j]);
        if (draw <= 0.0) {
          token = smp_index(s[j]);
          break;
        }
      }
    }
    *a.out = token;
    *a.ctr = 0u;
  }
  pdl_launch_dependents();
}

}  // namespace

int sample_grid(int n, int sm_count) {
  const int g = (n + SMP_MIN_SHARE - 1) / SMP_MIN_SHARE;
  return g < 1 ? 1 : g > sm_count ? sm_count : g > SAMPLE_MAX_GRID ? SAMPLE_MAX_GRID : g;
}

cudaError_t launch_sample(const SampleArgs &a, int sm_count, cudaStream_t s, bool pdl) {
  return launch_k(sample_kernel, dim3(sample_grid(a.n, sm_count)), dim3(SMP_THREADS), 0, s, pdl, a);
}

}  // namespace wgd

// ------------------------------------------------------------ stand-alone op
namespace wgd {
int api_fail(int code, const std::string &msg);
}

namespace {
struct SampleScratch {
  wgd::SampleParams *params = nullptr;
  double *uniform = nullptr;
  uint64_t *part = nullptr;
  unsigned *ctr = nullptr;
  int *out = nullptr;
  int sm = 0;
};
std::mutex g_smp_mu;
SampleScratch g_smp[16];
}  // namespace

#define CKS(x)                                                                                          \
  do {                                                                                                  \
    cudaError_t e_ = (x);                                                                               \
    if (e_ != cudaSuccess) return wgd::api_fail(WGD_ECUDA, std::string(#x) + ": " + cudaGetErrorString(e_)); \
  } while (0)

extern "C" int wgd_op_sample(const float *logits, int n, double temperature, int top_k, double top_p, double uniform,
                             int32_t *token_out, void *stream) {
  using namespace wgd;
  if (!logits || !token_out) return api_fail(WGD_EINVAL, "null argument");
  if (n < 1) return api_fail(WGD_EINVAL, "the logit row is empty");
  if (!(temperature >= 0 && temperature <= 2) || top_k < 1 || top_k > SAMPLE_MAX_K || !(top_p > 0 && top_p <= 1))
    return api_fail(WGD_EINVAL, "Invalid sampling settings.");
  if (!(uniform >= 0 && uniform < 1)) return api_fail(WGD_EINVAL, "the uniform draw must lie in [0, 1)");
  int dev = 0;
  CKS(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 16) return api_fail(WGD_EINVAL, "device index");
  std::lock_guard<std::mutex> lk(g_smp_mu);
  SampleScratch &S = g_smp[dev];
  if (!S.params) {
    cudaDeviceProp p;
    CKS(cudaGetDeviceProperties(&p, dev));
    S.sm = p.multiProcessorCount;
    CKS(cudaMalloc(&S.part, sizeof(uint64_t) * SAMPLE_MAX_GRID * SAMPLE_MAX_K));
    CKS(cudaMalloc(&S.ctr, sizeof(unsigned)));
    CKS(cudaMemset(S.ctr, 0, sizeof(unsigned)));
    CKS(cudaMalloc(&S.out, sizeof(int)));
    CKS(cudaMalloc(&S.uniform, sizeof(double)));
    CKS(cudaMalloc(&S.params, sizeof(SampleParams)));
  }
  cudaStream_t s = (cudaStream_t)stream;
  const SampleParams sp{temperature, top_p, top_k, 0};
  CKS(cudaMemcpyAsync(S.params, &sp, sizeof(sp), cudaMemcpyHostToDevice, s));
  CKS(cudaMemcpyAsync(S.uniform, &uniform, sizeof(double), cudaMemcpyHostToDevice, s));
  SampleArgs a{};
  a.logits = logits;
  a.n = n;
  a.params = S.params;
  a.uniform = S.uniform;
  a.out = S.out;
  a.part = S.part;
  a.ctr = S.ctr;
  CKS(launch_sample(a, S.sm, s, false));
  int32_t tok = -1;
  CKS(cudaMemcpyAsync(&tok, S.out, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  CKS(cudaStreamSynchronize(s));
  if (tok < 0) return api_fail(WGD_ENONFINITE, "Inference produced non-finite logits. Stop and report this model/runtime combination.");
  *token_out = tok;
  return WGD_OK;
}
