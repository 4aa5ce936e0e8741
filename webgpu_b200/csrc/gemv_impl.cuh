// Fused dequant GEMV for decode (batch <= 4 per pass), one instantiation set per
// GGML type (gemv_<type>.cu). Replaces the reference's matmulShader
// (shaders.ts:39-54 of the reference project: 64 threads per output row,
// byte-wise loads, one dispatch per weight page).
//
// Layout of work:
//   * A CTA is one "row group": W warps that split a row's 32-value units
//     (UPL units per lane, lanes of a warp on consecutive units, so each warp
//     instruction reads a contiguous span of quant bytes with 16-byte loads).
//   * Each lane keeps the activations of its units in registers for the whole
//     kernel (loaded once per CTA, optionally RMS-normalised on the way in).
//   * CTAs are persistent and take 4-row work items round-robin (the grid is
//     at most the resident capacity and the item count), so the tail is balanced
//     at 4-row granularity whatever the matrix shape; the first item's weight
//     rows are prefetched into L2 before the wait on the previous kernel.
//   * Per item, each warp reduces its 4*NB partial sums with a transposed
//     butterfly, the CTA combines warps in shared memory, and the epilogue
//     (store / residual add / SiLU / gated SiLU or GELU) writes the outputs.
#pragma once
#include "quant.cuh"
#include "kernels.h"

namespace wgd {

// Transposed butterfly: N partial values per lane -> lane holds the full warp
// sum of value index `idx` (lanes that share an index hold the same sum).
template <int N, int O>
struct TReduce {
  static __device__ __forceinline__ void run(float *v, int lane, int &idx) {
    if constexpr (N > 1) {
      constexpr int H = N / 2;
      const bool up = (lane & O) != 0;
#pragma unroll
      for (int i = 0; i < H; i++) {
        float keep = up ? v[i + H] : v[i];
        float send = up ? v[i] : v[i + H];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, O);
      }
      if (up) idx += H;
      if constexpr (O > 1) TReduce<H, O / 2>::run(v, lane, idx);
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], O);
      if constexpr (O > 1) TReduce<1, O / 2>::run(v, lane, idx);
    }
  }
};

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }
// shaders.ts:136 of the reference: 0.5*x*(1+tanh(0.7978845608*(x+0.044715*x^3)))
__device__ __forceinline__ float gelu_tanh_f(float x) {
  return 0.5f * x * (1.0f + tanhf(0.7978845608f * (x + 0.044715f * x * x * x)));
}

template <int T, int NB, int UPL>
__global__ void __launch_bounds__(256) gemv_kernel(const GemvArgs a) {
  constexpr int RB = GEMV_ROWS, V = RB * NB;
  __shared__ float red[2][8][V];
  __shared__ float s_norm[8][NB];
  __shared__ float s_inv[NB];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarp = blockDim.x >> 5;

  // Work items of 4 rows, round-robin over the CTAs (all resident; the grid never exceeds the
  // item count). The weights do not depend on earlier kernels: this CTA's first item goes to
  // L2 while the previous kernel finishes, and each later item while the one before it runs.
  const int items = (a.rows + RB - 1) / RB;
  auto prefetch_item = [&](int item) {
    for (int r = 0; r < RB; r++) {
      const int row = item * RB + r;
      if (row < a.rows)
        for (int off = tid * 16; off < a.drow; off += (int)blockDim.x * 16)
          asm volatile("prefetch.global.L2 [%0];" ::"l"(a.w + (int64_t)row * a.drow + off));
    }
  };
  prefetch_item((int)blockIdx.x);
  pdl_wait();

  // Activations of this lane's units, in registers for the whole kernel (the CTA's units cover
  // the whole row). One round of loads: x and, for the fused RMSNorm (normShader semantics:
  // x * rsqrt(mean(x^2)+eps) * w), its weight; the norm's sum of squares comes from the same
  // registers, and the 1/rms factor scales x*w once the CTA has the sum.
  XUnit xu[UPL][NB];
  int uidx[UPL];
  bool uval[UPL];
  float ss[NB];
#pragma unroll
  for (int b = 0; b < NB; b++) ss[b] = 0.f;
#pragma unroll
  for (int k = 0; k < UPL; k++) {
    const int u = (warp * UPL + k) * 32 + lane;
    uidx[k] = u;
    uval[k] = u < (a.cols >> 5);
    int ca = 0, cb = 0;
    if (uval[k]) Codec<T>::cols(u, ca, cb);
#pragma unroll
    for (int b = 0; b < NB; b++) {
      XUnit &X = xu[k][b];
      const bool live = uval[k] && b < a.batch;
      const float *xr = a.x + (int64_t)b * a.ldx;
#pragma unroll
      for (int i = 0; i < 16; i += 4) {
        float4 va = live ? __ldg(reinterpret_cast<const float4 *>(xr + ca + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
        float4 vb = live ? __ldg(reinterpret_cast<const float4 *>(xr + cb + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
        if (a.norm_w) {
          ss[b] = fmaf(va.x, va.x, fmaf(va.y, va.y, fmaf(va.z, va.z, fmaf(va.w, va.w, ss[b]))));
          ss[b] = fmaf(vb.x, vb.x, fmaf(vb.y, vb.y, fmaf(vb.z, vb.z, fmaf(vb.w, vb.w, ss[b]))));
          if (live) {
            const float4 wa = __ldg(reinterpret_cast<const float4 *>(a.norm_w + ca + i));
            const float4 wb = __ldg(reinterpret_cast<const float4 *>(a.norm_w + cb + i));
            va = make_float4(va.x * wa.x, va.y * wa.y, va.z * wa.z, va.w * wa.w);
            vb = make_float4(vb.x * wb.x, vb.y * wb.y, vb.z * wb.z, vb.w * wb.w);
          }
        }
        X.a[i] = va.x; X.a[i + 1] = va.y; X.a[i + 2] = va.z; X.a[i + 3] = va.w;
        X.b[i] = vb.x; X.b[i + 1] = vb.y; X.b[i + 2] = vb.z; X.b[i + 3] = vb.w;
      }
    }
  }
  if (a.norm_w) {
#pragma unroll
    for (int b = 0; b < NB; b++) {
      const float t = warp_sum(ss[b]);
      if (lane == 0) s_norm[warp][b] = t;
    }
    __syncthreads();
    if (tid < NB) {
      float t = 0.f;
      for (int w = 0; w < nwarp; w++) t += s_norm[w][tid];
      s_inv[tid] = rsqrtf(t / (float)a.cols + a.eps);
    }
  }
  __syncthreads();  // s_inv
#pragma unroll
  for (int k = 0; k < UPL; k++) {
#pragma unroll
    for (int b = 0; b < NB; b++) {
      XUnit &X = xu[k][b];
      const float inv = a.norm_w ? s_inv[b] : 1.f;
      float sa = 0.f, sb = 0.f;
#pragma unroll
      for (int i = 0; i < 16; i += 4) {
        if (a.norm_w) {
#pragma unroll
          for (int e = 0; e < 4; e++) { X.a[i + e] *= inv; X.b[i + e] *= inv; }
        }
        sa += (X.a[i] + X.a[i + 1]) + (X.a[i + 2] + X.a[i + 3]);
        sb += (X.b[i] + X.b[i + 1]) + (X.b[i + 2] + X.b[i + 3]);
      }
      X.sa = sa; X.sb = sb;
    }
  }
  pdl_launch_dependents();

  int buf = 0;
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    if (item + (int)gridDim.x < items) prefetch_item(item + (int)gridDim.x);
    const int row0 = item * RB;
    float acc[V];
#pragma unroll
    for (int v = 0; v < V; v++) acc[v] = 0.f;
#pragma unroll
    for (int r = 0; r < RB; r++) {
      const int row = row0 + r;
      if (row < a.rows) {
        const uint8_t *rp = a.w + (int64_t)row * a.drow;
#pragma unroll
        for (int k = 0; k < UPL; k++) {
          if (uval[k]) {
            Unit wu;
            Codec<T>::decode(rp, a.nb, uidx[k], wu);
#pragma unroll
            for (int b = 0; b < NB; b++) acc[r * NB + b] += unit_apply(wu, xu[k][b]);
          }
        }
      }
    }
    int vi = 0;
    TReduce<V, 16>::run(acc, lane, vi);
    if ((lane & (32 / V - 1)) == 0) red[buf][warp][vi] = acc[0];
    __syncthreads();
    if (tid < V) {
      float val = 0.f;
      for (int w = 0; w < nwarp; w++) val += red[buf][w][tid];
      const int r = tid / NB, b = tid % NB;
      const int row = row0 + r;
      if (b < a.batch) {
        if (a.epi == EPI_GLU_SILU || a.epi == EPI_GLU_GELU) {
          if (r < RB / 2 && row < a.rows) {
            float up = 0.f;
            for (int w = 0; w < nwarp; w++) up += red[buf][w][(r + RB / 2) * NB + b];
            const float g = a.epi == EPI_GLU_SILU ? silu_f(val) : gelu_tanh_f(val);
            a.y[(int64_t)b * a.ldy + item * (RB / 2) + r] = g * up;
          }
        } else if (row < a.rows) {
          if (a.bias) val += __ldg(a.bias + row);
          float *dst = a.y + (int64_t)b * a.ldy + row;
          if (a.epi == EPI_ADD) *dst = __ldcg(dst) + val;  // through L2: see the end of the kernel
          else if (a.epi == EPI_SILU) *dst = silu_f(val);
          else *dst = val;
        }
      }
    }
    buf ^= 1;
  }
  // Under programmatic dependent launch the next kernel's CTAs may already be resident on this
  // SM, past the point where a kernel boundary would have invalidated its L1, so no line of an
  // output that other SMs update may stay in this SM's L1: residual reads go through L2 (above),
  // and the device-scope fence at the end also invalidates the L1 (without it a Q8_0 model's
  // logits came out 12-25 % off).
  __syncthreads();
  if (tid == 0) __threadfence();
}

template <int T, int NB, int UPL>
cudaError_t launch_gemv_cfg(const GemvArgs &a, cudaStream_t s, bool pdl, int sm_count) {
  const int units = a.cols / 32;
  const int wpr = (units + 32 * UPL - 1) / (32 * UPL);
  if (wpr > 8) return cudaErrorInvalidValue;
  static int occ = -1;
  if (occ < 0) {
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gemv_kernel<T, NB, UPL>, 32 * wpr, 0);
    if (e != cudaSuccess || occ < 1) occ = 1;
  }
  const int items = (a.rows + GEMV_ROWS - 1) / GEMV_ROWS;
  int grid = sm_count * occ;
  if (grid > items) grid = items;
  if (grid < 1) grid = 1;
  return launch_k(gemv_kernel<T, NB, UPL>, dim3(grid), dim3(32 * wpr), 0, s, pdl, a);
}

// Chooses the register footprint for this width/batch: units per lane (UPL)
// and the batch chunk NB, with at most 8 warps per CTA.
template <int T>
cudaError_t launch_gemv_type(const GemvArgs &a, cudaStream_t s, bool pdl, int sm_count) {
  const int units = a.cols / 32;
  if (a.batch == 1) {
    if (units <= 8 * 32 * 2) return launch_gemv_cfg<T, 1, 2>(a, s, pdl, sm_count);
    return launch_gemv_cfg<T, 1, 3>(a, s, pdl, sm_count);
  }
  if (a.batch == 2) {
    if (units <= 8 * 32) return launch_gemv_cfg<T, 2, 1>(a, s, pdl, sm_count);
    return launch_gemv_cfg<T, 2, 2>(a, s, pdl, sm_count);
  }
  return launch_gemv_cfg<T, 4, 1>(a, s, pdl, sm_count);
}

}  // namespace wgd
