// Shared device/host helpers for the wgd library (sm_100a only).
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string>
#include <utility>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "wgd is built for sm_100a (Blackwell B200) only"
#endif

namespace wgd {

// GGML tensor types the reference decodes (gguf.ts:6-11 of the reference project).
enum GgmlType : int { F32 = 0, F16 = 1, Q4_0 = 2, Q8_0 = 8, Q4_K = 12, Q5_K = 13, Q6_K = 14 };

inline int block_elems(int t) { return t == F32 || t == F16 ? 1 : (t == Q4_0 || t == Q8_0) ? 32 : 256; }
inline int block_bytes(int t) {
  switch (t) {
    case F32: return 4; case F16: return 2; case Q4_0: return 18; case Q8_0: return 34;
    case Q4_K: return 144; case Q5_K: return 176; case Q6_K: return 210; default: return 0;
  }
}
inline bool type_supported(int t) { return block_bytes(t) != 0; }
inline int64_t gguf_row_bytes(int t, int64_t cols) { return cols / block_elems(t) * block_bytes(t); }
inline int64_t align_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

// Device row layout: every row starts 16-byte aligned.
//   F32/F16     : the values, padded.
//   Q4_0 / Q8_0 : [nb x 16|32 B quants][nb x 2 B fp16 d], padded.
//   Q4_K / Q5_K : the GGUF super-blocks unchanged (144 / 176 B are multiples of 16).
//   Q6_K        : [nsb x 208 B (ql 128, qh 64, scales 16)][nsb x 2 B fp16 d], padded.
// The bytes are the GGUF bytes, moved; only the row padding is added.
inline int64_t dev_row_bytes(int t, int64_t cols) { return align_up(gguf_row_bytes(t, cols), 16); }

// ------------------------------------------------------------------ device

__device__ __forceinline__ float h2f(uint32_t bits16) {
  return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xffffu)));
}

__device__ __forceinline__ uint4 ldg_stream(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ldg_cached(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ldg_u32(const void *p) {
  uint32_t v;
  asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ldg_u16(const void *p) {
  unsigned short v;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

// Programmatic dependent launch: the dependent grid may start its prologue
// (weight prefetch) while this grid drains; it waits here for our results.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Base-254 digits of t in [-127, 127]: a = rint(t), b = rint((t - a) * 254),
// c = rint(((t - a) * 254 - b) * 254), each as a two's-complement byte in the low 8 bits.
// Rounding to the nearest integer (ties to even) of |x| < 2^22 is (x + 1.5*2^23) - 1.5*2^23,
// and the integer sits in the low mantissa bits of x + 1.5*2^23: additions only, no
// float->int conversion (those issue at a quarter of the FMA rate). Every step is an
// explicit round-to-nearest operation, so no multiply-add is contracted.
__device__ __forceinline__ void digits254(float t, uint32_t &a, uint32_t &b, uint32_t &c) {
  const float M = 12582912.f;
  const float ta = __fadd_rn(t, M), r1 = __fmul_rn(__fsub_rn(t, __fsub_rn(ta, M)), 254.f);
  const float tb = __fadd_rn(r1, M), r2 = __fmul_rn(__fsub_rn(r1, __fsub_rn(tb, M)), 254.f);
  const float tc = __fadd_rn(r2, M);
  a = __float_as_uint(ta) & 255u;
  b = __float_as_uint(tb) & 255u;
  c = __float_as_uint(tc) & 255u;
}

// PRMT-based nibble/byte to float: 0x3F00_qq00_00 pattern gives 0.5 + q/256 for
// q in [0, 255] placed in byte 2, i.e. an exact affine image of q. Summing
// f*x and correcting with 0.5*sum(x) recovers sum(q*x) with fp32 rounding only.
__device__ __forceinline__ float byte_as_affine(uint32_t word, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(word), "r"(0x3Fu), "r"(sel));
  return __uint_as_float(r);
}
// selector placing byte k of `word` into byte 2 and 0x3F (byte 0 of the second
// operand, index 4) into byte 3; bytes 0,1 from index 5 (zero).
__host__ __device__ constexpr uint32_t sel_byte(int k) { return 0x4055u | ((uint32_t)k << 8); }

}  // namespace wgd

namespace wgd {
// Kernel launch with optional programmatic dependent launch (the kernel must
// call pdl_wait() before it reads anything an earlier kernel wrote).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                            Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
}  // namespace wgd
