// Tensor-parallel exchange over peer-mapped device memory (CUDA IPC between the
// processes of one node; NVLink/NVSwitch carries the stores).
//
// Every rank owns one exchange buffer. A collective pushes this rank's data
// with plain stores into every peer's buffer (slot = this rank), publishes a
// per-CTA flag carrying the collective's epoch (a device-side counter that all
// ranks advance identically, so CUDA graphs can replay the sequence), waits for
// the peers' flags with a bounded spin, and reduces its own slots in rank order
// (the same order on every rank, so the result is bit-identical everywhere).
// Slots are double-buffered by epoch parity: a rank can only push collective
// e+2 after every peer has entered e+1, i.e. finished reading e.
// A wait that runs out sets an error word (read by the host after the forward)
// and lets the kernel finish; nothing traps.
#include <algorithm>
#include <cstring>
#include "common.cuh"
#include "tp.h"

namespace wgd {

constexpr int TP_MAX = 8, TP_CTAS = 32;

struct Header {
  unsigned epoch, done, err, pad[29];
};

// Byte offsets inside an exchange buffer.
struct Layout {
  size_t flags, aflags, gflags, am, slots, gather, total;
  size_t cap, gcap;
  size_t pbar, pcand, pslot;  // the persistent kernel's region
};
// persistent kernel region: arrival counter (own 256-byte line), candidate tables
// [2 token parities][TP_MAX ranks][256] (float2), partial-row slots [2][TP_MAX][16384] floats
// (16384 = the widest hidden size the configuration allows)
constexpr size_t P_CAND_SLOTS = 256, P_SLOT_FLOATS = 16384;
static Layout make_layout(size_t cap, size_t gcap) {
  Layout L{};
  size_t o = sizeof(Header);
  L.flags = o; o += sizeof(unsigned) * TP_MAX * TP_CTAS;
  L.gflags = o; o += sizeof(unsigned) * TP_MAX * TP_CTAS;
  L.aflags = o; o += sizeof(unsigned) * TP_MAX;
  o = (o + 255) / 256 * 256;
  L.am = o; o += sizeof(float) * 2 * TP_MAX;
  o = (o + 255) / 256 * 256;
  L.slots = o; o += sizeof(float) * 2 * TP_MAX * cap;
  L.gather = o; o += sizeof(float) * gcap;
  o = (o + 255) / 256 * 256;
  L.pbar = o; o += 256;
  L.pcand = o; o += sizeof(float) * 2 * 2 * TP_MAX * P_CAND_SLOTS;
  o = (o + 255) / 256 * 256;
  L.pslot = o; o += sizeof(float) * 2 * TP_MAX * P_SLOT_FLOATS;
  L.total = (o + 255) / 256 * 256;
  L.cap = cap;
  L.gcap = gcap;
  return L;
}

struct TpDev {
  char *buf[TP_MAX];  // every rank's exchange buffer (own included), mapped here
  int rank, size;
  size_t flags, aflags, gflags, am, slots, gather, cap;
};

struct TpComm {
  int rank = 0, size = 1;
  Layout L{};
  char *local = nullptr;
  char *peer[TP_MAX] = {nullptr};
  bool opened = false;
  TpDev dev{};
};

int tp_handle_size() { return (int)sizeof(cudaIpcMemHandle_t); }

static int err_out(std::string *err, const std::string &m, int code = 3) {
  if (err) *err = m;
  return code;
}

int tp_create(TpComm **out, int rank, int size, size_t max_floats, std::string *err) {
  auto *t = new TpComm();
  t->rank = rank;
  t->size = size;
  // The gather area holds a full vocabulary row; 1M floats covers the reference's vocab limit.
  t->L = make_layout((max_floats + 3) / 4 * 4, 1u << 20);
  if (cudaMalloc(&t->local, t->L.total) != cudaSuccess || cudaMemset(t->local, 0, t->L.total) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess) {
    delete t;
    return err_out(err, "exchange buffer allocation failed");
  }
  *out = t;
  return 0;
}

int tp_export(TpComm *t, void *handle_out, std::string *err) {
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, t->local);
  if (e != cudaSuccess) return err_out(err, std::string("cudaIpcGetMemHandle: ") + cudaGetErrorString(e));
  memcpy(handle_out, &h, sizeof(h));
  return 0;
}

int tp_open(TpComm *t, const void *handles, std::string *err) {
  if (t->opened) return 0;
  const char *hs = (const char *)handles;
  for (int j = 0; j < t->size; j++) {
    if (j == t->rank) { t->peer[j] = t->local; continue; }
    cudaIpcMemHandle_t h;
    memcpy(&h, hs + j * sizeof(h), sizeof(h));
    void *p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return err_out(err, std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
    t->peer[j] = (char *)p;
  }
  TpDev &d = t->dev;
  for (int j = 0; j < TP_MAX; j++) d.buf[j] = j < t->size ? t->peer[j] : nullptr;
  d.rank = t->rank;
  d.size = t->size;
  d.flags = t->L.flags;
  d.aflags = t->L.aflags;
  d.gflags = t->L.gflags;
  d.am = t->L.am;
  d.slots = t->L.slots;
  d.gather = t->L.gather;
  d.cap = t->L.cap;
  t->opened = true;
  return 0;
}

void tp_destroy(TpComm *t) {
  if (!t) return;
  for (int j = 0; j < t->size; j++)
    if (j != t->rank && t->peer[j]) cudaIpcCloseMemHandle(t->peer[j]);
  if (t->local) cudaFree(t->local);
  delete t;
}

bool tp_failed(TpComm *t) {
  Header h;
  if (cudaMemcpy(&h, t->local, sizeof(h), cudaMemcpyDeviceToHost) != cudaSuccess) return true;
  return h.err != 0;
}

// ------------------------------------------------------------------ device

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(unsigned *p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ Header *hdr(const TpDev &d, int j) { return reinterpret_cast<Header *>(d.buf[j]); }

// Bounded wait until *p >= e; records a timeout in the local header.
__device__ bool wait_flag(const TpDev &d, const unsigned *p, unsigned e, unsigned long long limit) {
  for (unsigned long long i = 0; i < limit; i++) {
    if ((int)(ld_acquire(p) - e) >= 0) return true;
    __nanosleep(64);
  }
  atomicExch(&hdr(d, d.rank)->err, 1u);
  return false;
}

__device__ __forceinline__ void finish(const TpDev &d, unsigned e) {
  __syncthreads();
  if (threadIdx.x == 0) {
    Header *h = hdr(d, d.rank);
    if (atomicAdd(&h->done, 1u) == gridDim.x - 1) {
      h->done = 0;
      __threadfence();
      atomicExch(&h->epoch, e);
    }
  }
}

__global__ void allreduce_kernel(const TpDev d, const float *partial, float *out, size_t n, int add, unsigned long long limit) {
  __shared__ unsigned e_s;
  pdl_wait();
  if (threadIdx.x == 0) e_s = *(volatile unsigned *)&hdr(d, d.rank)->epoch + 1u;
  __syncthreads();
  const unsigned e = e_s;
  const int par = e & 1, c = blockIdx.x;
  const size_t chunk = (n + gridDim.x - 1) / gridDim.x;
  const size_t lo = (size_t)c * chunk, hi = lo + chunk < n ? lo + chunk : n;
  // push this rank's slice into slot [par][rank] of every rank
  for (int j = 0; j < d.size; j++) {
    float *dst = reinterpret_cast<float *>(d.buf[j] + d.slots) + ((size_t)par * TP_MAX + d.rank) * d.cap;
    for (size_t i = lo + threadIdx.x; i < hi; i += blockDim.x) dst[i] = partial[i];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int j = 0; j < d.size; j++) st_release(reinterpret_cast<unsigned *>(d.buf[j] + d.flags) + d.rank * TP_CTAS + c, e);
    for (int j = 0; j < d.size; j++)
      wait_flag(d, reinterpret_cast<const unsigned *>(d.buf[d.rank] + d.flags) + j * TP_CTAS + c, e, limit);
    __threadfence();
  }
  __syncthreads();
  const float *slots = reinterpret_cast<const float *>(d.buf[d.rank] + d.slots) + (size_t)par * TP_MAX * d.cap;
  for (size_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    float s = 0.f;
    for (int j = 0; j < d.size; j++) s += __ldcg(slots + (size_t)j * d.cap + i);
    out[i] = add ? __ldcg(out + i) + s : s;  // residual read through L2
  }
  finish(d, e);
  pdl_launch_dependents();
}

__global__ void argmax_gather_kernel(const TpDev d, int *idx, float *val, int vocab0, unsigned long long limit) {
  pdl_wait();
  if (threadIdx.x != 0) return;
  const unsigned e = *(volatile unsigned *)&hdr(d, d.rank)->epoch + 1u;
  const int li = *idx;
  const float lv = *val;
  for (int j = 0; j < d.size; j++) {
    float *am = reinterpret_cast<float *>(d.buf[j] + d.am) + 2 * d.rank;
    am[0] = lv;
    am[1] = __int_as_float(li < 0 ? -1 : li + vocab0);
  }
  __threadfence_system();
  for (int j = 0; j < d.size; j++) st_release(reinterpret_cast<unsigned *>(d.buf[j] + d.aflags) + d.rank, e);
  for (int j = 0; j < d.size; j++) wait_flag(d, reinterpret_cast<const unsigned *>(d.buf[d.rank] + d.aflags) + j, e, limit);
  __threadfence();
  const float *am = reinterpret_cast<const float *>(d.buf[d.rank] + d.am);
  float bv = 0.f;
  int bi = -1;
  for (int j = 0; j < d.size; j++) {
    const float v = __ldcg(am + 2 * j);
    const int i = __float_as_int(__ldcg(am + 2 * j + 1));
    if (i >= 0 && (bi < 0 || v > bv || (v == bv && i < bi))) { bv = v; bi = i; }
  }
  *idx = bi;
  *val = bv;
  atomicExch(&hdr(d, d.rank)->epoch, e);
}


// First vocabulary row of rank j: the vocabulary is split in whole 16-row tiles (the LM head's
// tile layout), rank j owning tiles [tiles*j/size, tiles*(j+1)/size).
__device__ __forceinline__ int vocab_lo(int total, int j, int size) {
  const int tiles = (total + 15) / 16;
  const int lo = (int)((long long)tiles * j / size) * 16;
  return lo < total ? lo : total;
}

__global__ void gather_rows_kernel(const TpDev d, float *rows, int total, unsigned long long limit) {
  __shared__ unsigned e_s;
  pdl_wait();
  if (threadIdx.x == 0) e_s = *(volatile unsigned *)&hdr(d, d.rank)->epoch + 1u;
  __syncthreads();
  const unsigned e = e_s;
  const int c = blockIdx.x;
  // push my slice c
  {
    const int lo = vocab_lo(total, d.rank, d.size), hi = vocab_lo(total, d.rank + 1, d.size), cnt = hi - lo;
    const int ch = (cnt + gridDim.x - 1) / gridDim.x, a = lo + c * ch, b = min(hi, a + ch);
    for (int j = 0; j < d.size; j++) {
      float *g = reinterpret_cast<float *>(d.buf[j] + d.gather);
      for (int i = a + threadIdx.x; i < b; i += blockDim.x) g[i] = rows[i];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int j = 0; j < d.size; j++) st_release(reinterpret_cast<unsigned *>(d.buf[j] + d.gflags) + d.rank * TP_CTAS + c, e);
    for (int j = 0; j < d.size; j++)
      wait_flag(d, reinterpret_cast<const unsigned *>(d.buf[d.rank] + d.gflags) + j * TP_CTAS + c, e, limit);
    __threadfence();
  }
  __syncthreads();
  const float *g = reinterpret_cast<const float *>(d.buf[d.rank] + d.gather);
  for (int j = 0; j < d.size; j++) {
    const int lo = vocab_lo(total, j, d.size), hi = vocab_lo(total, j + 1, d.size), cnt = hi - lo;
    const int ch = (cnt + gridDim.x - 1) / gridDim.x, a = lo + c * ch, b = min(hi, a + ch);
    for (int i = a + threadIdx.x; i < b; i += blockDim.x) rows[i] = __ldcg(g + i);
  }
  finish(d, e);
}

int tp_persist_view(TpComm *t, TpPersistView *out, std::string *err) {
  if (!t || !t->opened) return err_out(err, "tensor-parallel peers are not open (call wgd_tp_open_peers)", 6);
  for (int j = 0; j < TP_MAX; j++) out->buf[j] = j < t->size ? t->peer[j] : nullptr;
  out->bar = t->L.pbar;
  out->cand = t->L.pcand;
  out->slot = t->L.pslot;
  return 0;
}

static unsigned long long limit_or_default(unsigned long long l) { return l ? l : (1ull << 25); }

int tp_allreduce_add(TpComm *t, const float *partial, float *hidden, size_t n, cudaStream_t s, unsigned long long spin_limit,
                     std::string *err) {
  if (!t->opened) return err_out(err, "tensor-parallel peers are not open (call wgd_tp_open_peers)", 6);
  if (n > t->L.cap) return err_out(err, "allreduce larger than the exchange slots", 1);
  cudaError_t e = launch_k(allreduce_kernel, dim3(TP_CTAS), dim3(256), 0, s, true, t->dev, partial, hidden, n, 1,
                           limit_or_default(spin_limit));
  return e == cudaSuccess ? 0 : err_out(err, std::string("allreduce launch: ") + cudaGetErrorString(e));
}

int tp_allreduce_inplace(TpComm *t, float *buf, size_t n, cudaStream_t s, unsigned long long spin_limit, std::string *err) {
  if (!t->opened) return err_out(err, "tensor-parallel peers are not open (call wgd_tp_open_peers)", 6);
  if (n > t->L.cap) return err_out(err, "allreduce larger than the exchange slots", 1);
  cudaError_t e = launch_k(allreduce_kernel, dim3(TP_CTAS), dim3(256), 0, s, true, t->dev, (const float *)buf, buf, n, 0,
                           limit_or_default(spin_limit));
  return e == cudaSuccess ? 0 : err_out(err, std::string("allreduce launch: ") + cudaGetErrorString(e));
}

int tp_argmax_gather(TpComm *t, int *idx, float *val, int vocab0, cudaStream_t s, unsigned long long spin_limit, std::string *err) {
  if (!t->opened) return err_out(err, "tensor-parallel peers are not open (call wgd_tp_open_peers)", 6);
  cudaError_t e = launch_k(argmax_gather_kernel, dim3(1), dim3(32), 0, s, true, t->dev, idx, val, vocab0, limit_or_default(spin_limit));
  return e == cudaSuccess ? 0 : err_out(err, std::string("argmax gather launch: ") + cudaGetErrorString(e));
}

int tp_gather_rows(TpComm *t, float *rows, int total, int vocab0, int count, cudaStream_t s, unsigned long long spin_limit,
                   std::string *err) {
  // the kernel derives every rank's rows from the tile rule; they must agree with the caller's shard
  const int tiles = (total + 15) / 16;
  const int lo = std::min(total, (int)((long long)tiles * t->rank / t->size) * 16);
  const int hi = std::min(total, (int)((long long)tiles * (t->rank + 1) / t->size) * 16);
  if (lo != vocab0 || hi - lo != count) return err_out(err, "vocabulary shard does not follow the 16-row tile split", 1);
  if (!t->opened) return err_out(err, "tensor-parallel peers are not open (call wgd_tp_open_peers)", 6);
  if ((size_t)total > t->L.gcap) return err_out(err, "gather larger than the exchange area", 1);
  cudaError_t e = launch_k(gather_rows_kernel, dim3(TP_CTAS), dim3(256), 0, s, true, t->dev, rows, total, limit_or_default(spin_limit));
  return e == cudaSuccess ? 0 : err_out(err, std::string("gather launch: ") + cudaGetErrorString(e));
}

}  // namespace wgd
