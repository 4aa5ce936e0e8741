// Fused dequant GEMV for decode (batch <= 4 per pass), one instantiation set per
// GGML type (gemv_<type>.cu). Replaces the reference's matmulShader
// (shaders.ts:68-83 of the reference project: 64 threads per output row,
// byte-wise loads, one dispatch per weight page).
//
// Layout of work:
//   * A CTA is one "row group": W warps that split a row's 32-value units
//     (UPL units per lane, lanes of a warp on consecutive units, so each warp
//     instruction reads a contiguous span of quant bytes with 16-byte loads).
//   * Each lane keeps the activations of its units in registers for the whole
//     kernel (loaded once per CTA, optionally RMS-normalised on the way in).
//   * CTAs are persistent and pull 4-row work items from a ticket counter, so
//     the tail is balanced at 4-row granularity whatever the matrix shape.
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
// shaders.ts:165 of the reference: 0.5*x*(1+tanh(0.7978845608*(x+0.044715*x^3)))
__device__ __forceinline__ float gelu_tanh_f(float x) {
  return 0.5f * x * (1.0f + tanhf(0.7978845608f * (x + 0.044715f * x * x * x)));
}

template <int T, int NB, int UPL>
__global__ void __launch_bounds__(256) gemv_kernel(const GemvArgs a) {
  constexpr int RB = GEMV_ROWS, V = RB * NB;
  __shared__ float red[2][8][V];
  __shared__ float s_norm[8][NB];
  __shared__ float s_inv[NB];
  __shared__ int s_item[2];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarp = blockDim.x >> 5;

  pdl_wait();
  if (tid == 0) s_item[0] = (int)atomicAdd(a.ctr, 1u);

  // Fused RMSNorm of the activation rows (normShader semantics: x * rsqrt(mean(x^2)+eps) * w).
  if (a.norm_w) {
#pragma unroll
    for (int b = 0; b < NB; b++) {
      float s = 0.f;
      if (b < a.batch) {
        const float4 *xr = reinterpret_cast<const float4 *>(a.x + (int64_t)b * a.ldx);
        for (int c = tid; c < (a.cols >> 2); c += blockDim.x) {
          float4 v = __ldg(xr + c);
          s = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, s))));
        }
      }
      s = warp_sum(s);
      if (lane == 0) s_norm[warp][b] = s;
    }
    __syncthreads();
    if (tid < NB) {
      float t = 0.f;
      for (int w = 0; w < nwarp; w++) t += s_norm[w][tid];
      s_inv[tid] = rsqrtf(t / (float)a.cols + a.eps);
    }
  }
  __syncthreads();

  // Activations of this lane's units, in registers for the whole kernel.
  XUnit xu[UPL][NB];
  int uidx[UPL];
  bool uval[UPL];
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
      float sa = 0.f, sb = 0.f;
      const bool live = uval[k] && b < a.batch;
      const float *xr = a.x + (int64_t)b * a.ldx;
      const float inv = a.norm_w ? s_inv[b] : 1.f;
#pragma unroll
      for (int i = 0; i < 16; i += 4) {
        float4 va = live ? __ldg(reinterpret_cast<const float4 *>(xr + ca + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
        float4 vb = live ? __ldg(reinterpret_cast<const float4 *>(xr + cb + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
        if (a.norm_w && live) {
          float4 wa = __ldg(reinterpret_cast<const float4 *>(a.norm_w + ca + i));
          float4 wb = __ldg(reinterpret_cast<const float4 *>(a.norm_w + cb + i));
          va = make_float4(va.x * inv * wa.x, va.y * inv * wa.y, va.z * inv * wa.z, va.w * inv * wa.w);
          vb = make_float4(vb.x * inv * wb.x, vb.y * inv * wb.y, vb.z * inv * wb.z, vb.w * inv * wb.w);
        }
        X.a[i] = va.x; X.a[i + 1] = va.y; X.a[i + 2] = va.z; X.a[i + 3] = va.w;
        X.b[i] = vb.x; X.b[i + 1] = vb.y; X.b[i + 2] = vb.z; X.b[i + 3] = vb.w;
        sa += (va.x + va.y) + (va.z + va.w);
        sb += (vb.x + vb.y) + (vb.z + vb.w);
      }
      X.sa = sa; X.sb = sb;
    }
  }
  pdl_launch_dependents();

  const int items = (a.rows + RB - 1) / RB;
  int buf = 0;
  int item = s_item[0];
  while (item < items) {
    if (tid == 0) s_item[buf ^ 1] = (int)atomicAdd(a.ctr, 1u);
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
          if (a.epi == EPI_ADD) *dst += val;
          else if (a.epi == EPI_SILU) *dst = silu_f(val);
          else *dst = val;
        }
      }
    }
    item = s_item[buf ^ 1];
    buf ^= 1;
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(a.ctr + 1, 1u) == gridDim.x - 1) {
      a.ctr[0] = 0u;
      a.ctr[1] = 0u;
    }
  }
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
