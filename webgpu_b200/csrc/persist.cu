// Persistent decode kernel (see persist.h). Per token it runs, for every
// layer, the phases of PagedEngine.forward's denseLayer (engine.ts:217-251 of
// the reference): RMSNorm+QKV projection (+bias), RoPE + KV ring write +
// attention (attentionShader, shaders.ts:88-122), output projection +
// residual, RMSNorm + gate|up projection + SwiGLU, down projection +
// residual; then the final norm + LM head and the greedy argmax
// (engine.ts:305-309), and feeds the token back to the embedding gather
// (engine.ts:140-145).
//
// Synchronisation:
//  * between phases, a grid barrier (all CTAs are co-resident: cooperative
//    launch, one CTA per SM) with one arrival counter that only grows;
//  * inside a CTA, the producer warp and the consumer warps share a ring of
//    shared-memory slots guarded by mbarriers ("full": transaction bytes of the
//    bulk copy; "empty": the epilogue warp's arrival once every compute warp has
//    reported the stage done);
//  * each CTA owns whole 16-row output tiles; the compute warps hand each
//    chunk's 16 row sums to the epilogue warp through a ring of result stages
//    (mbarrier "done", one arrival per compute warp), and the epilogue warp adds
//    a tile's chunks in k-block order, so every sum has a fixed order. A result
//    stage is free again without a barrier of its own: stage g + ns of the
//    weight ring is only issued after the epilogue warp has read the results of
//    stage g, and ns <= P_RES_STAGES;
//  * tensor parallel, after a phase whose outputs are pushed to the peers (O,
//    down) and after the LM head, a two-level cross-rank barrier (x_sync)
//    replaces the grid barrier.
// Every wait is bounded by a globaltimer deadline; a wait that runs out sets
// status[0] = 1 and the whole grid winds down (the producer first waits for its
// copies in flight).
#include <float.h>

#include "gemv2_impl.cuh"
#include "kernels.h"
#include "persist.h"
#include "quant.cuh"
#include "tile.cuh"

namespace wgd {
namespace {

// ------------------------------------------------------------------ PTX helpers

__device__ __forceinline__ uint32_t su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t *b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t *b, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(su32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Blocking form: the hardware suspends the thread until the phase completes or a
// hardware time limit passes (then false).
__device__ __forceinline__ bool mbar_try(uint64_t *b, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(su32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// bulk copy global -> this CTA's shared memory, completing on mbarrier `bar`
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(su32(dst)),
               "l"(src), "r"(bytes), "r"(su32(bar))
               : "memory");
}
__device__ __forceinline__ uint64_t gtime() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void cp_async16(void *smem, const void *g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(su32(smem)), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

constexpr uint64_t P_TIMEOUT_NS = 2000000000ull;  // 2 s: far above any legitimate wait

// Phase timeline for profiling builds (-DWGD_PERSIST_TRACE): globaltimer stamps of
// CTAs 0 and 100 per (step, phase): [0] start, [1] input digitised, [2] last unit
// computed, [3] finished; [4], [5] producer issue of the phase's first / last stage.
#ifdef WGD_PERSIST_TRACE
constexpr int TR_STEPS = 4, TR_PHASES = 256, TR_SLOTS = 8;
__device__ uint64_t g_trace[2][TR_STEPS][TR_PHASES][TR_SLOTS];
// every CTA's barrier arrival / release of step 1: [cta][barrier index][2]
constexpr int TR_BARS = 256;
__device__ uint64_t g_bars[160][TR_BARS][2];
__device__ int g_bar_index[160];
__device__ uint64_t g_wait_acc[2];  // ns thread 0 of CTAs 0 / 100 spent waiting for ring slots (per phase)
#define P_TRACE(step, phase, slot)                                                                          \
  do {                                                                                                     \
    if ((blockIdx.x == 0 || blockIdx.x == 100) && (step) < TR_STEPS && (phase) < TR_PHASES)                \
      g_trace[blockIdx.x == 0 ? 0 : 1][step][phase][slot] = gtime();                                       \
  } while (0)
#else
#define P_TRACE(step, phase, slot) \
  do {                             \
  } while (0)
#endif

// Warp roles: 0..13 compute (digitise, tile-chunk math, attention, embedding), 14 epilogue
// (sums each tile's chunk results in k-block order, stores, greedy tracking), 15 producer.
constexpr int P_EWARP = P_CWARPS, P_PWARP = P_CWARPS + 1;
constexpr int P_MAXSTAGES = 8, P_STAGE_UNITS = 16, P_RES_STAGES = 8;
static_assert(P_MAXSTAGES <= P_RES_STAGES, "a result stage is recycled through the weight ring (ns <= P_RES_STAGES)");
static_assert(P_SLOT_BYTES / 2304 <= P_CWARPS && P_SLOT_BYTES / 2304 <= P_STAGE_UNITS, "a stage holds at most one chunk per compute warp");

// Shared state of one CTA besides the ring and the xs region.
struct PShared {
  float res[P_RES_STAGES][P_STAGE_UNITS][16];  // per stage (mod P_RES_STAGES): the 16 row sums of each chunk
  float red[P_CWARPS];
  int dsum[P_CWARPS][48];  // digitiser scratch: one super-block's digit sums per warp
  float2 best[P_CWARPS + 1];
  PPhase dsc[3];  // phase descriptors, a ring over the phase sequence: q, q + 1 (look-ahead), q + 2 (being copied)
  int flags[4];  // [0] stop (finished / winding down), [1] attention last-arriver, [2] token, [3] stop snapshot
};
// compute + epilogue warps / compute warps only
__device__ __forceinline__ void bar_all() { asm volatile("bar.sync 1, %0;" ::"n"((P_CWARPS + 1) * 32) : "memory"); }
__device__ __forceinline__ void bar_comp() { asm volatile("bar.sync 3, %0;" ::"n"(P_CWARPS * 32) : "memory"); }

__device__ __forceinline__ int chunk_bytes(int type) { return type == Q4_K ? 2304 : 3360; }
__device__ __forceinline__ int slot_units(int type) { return P_SLOT_BYTES / chunk_bytes(type); }

// CTA c owns whole output tiles [tiles*c/grid, tiles*(c+1)/grid): no tile is cut between CTAs, so
// each output is summed in k order by one CTA with no cross-CTA reduction. (A partition into equal
// unit counts with the cut tiles finished by their first CTA was measured: the fix-up's L2 round
// trips at the end of every phase cost more than the balance gained, 733 vs 656 us per token on the
// 8-layer model.)
__device__ __forceinline__ void unit_range(int tiles, int nkb, int grid, int c, int &u0, int &u1) {
  u0 = (int)((long long)tiles * c / grid) * nkb;
  u1 = (int)((long long)tiles * (c + 1) / grid) * nkb;
}

// better(a, b): a is a finite logit with a higher value, or equal value and lower index
__device__ __forceinline__ bool better(float va, int ia, float vb, int ib) {
  if (ia < 0) return false;
  if (ib < 0) return true;
  return va > vb || (va == vb && ia < ib);
}

// ------------------------------------------------------------------ GEMV pieces

// Digit records of the phase input in shared memory (one activation row), laid
// out so that the 16-byte loads of a warp hit distinct bank groups: per 256-column
// super-block sb,
//   brec sb*960 + (dg*4 + tig)*80 + j*8 + hi*4   digit plane dg at k = 4tig.. (hi 0) /
//                                                16+4tig.. (hi 1) of 32-block j
//   dsw  sb*256 + lane*8                         the lane's B fragment words (low bytes, high
//                                                bytes) of the digit sums of MMA column grp = dg:
//                                                Q4_K: 32-block sums j = 4tig..4tig+3 (tig < 2);
//                                                Q6_K: 16-run sums r = 4tig..4tig+3; zero elsewhere
//   sxs[sb]                                      digit scale
// (records 80 bytes apart: 12 live records fall on 8 bank groups, two wavefronts).
struct PX {
  uint8_t *brec, *dsw;
  float *sxs;
};
__host__ __device__ inline size_t px_bytes(int cols) {
  const size_t nsb = (size_t)cols / 256;
  return nsb * 960 + nsb * 256 + nsb * 4 + 64;
}
__device__ __forceinline__ PX px_carve(uint8_t *xs, int cols) {
  const int nsb = cols >> 8;
  PX X;
  X.brec = xs;
  X.dsw = xs + (size_t)nsb * 960;
  X.sxs = reinterpret_cast<float *>(X.dsw + (size_t)nsb * 256);
  return X;
}
constexpr int P_MAXSBW = 5;  // super-blocks per compute warp: inputs up to 14*5*256 = 17920 wide
static_assert(P_CWARPS * P_MAXSBW * 256 >= 16384, "digit records must cover 16384-wide inputs");

// Lane constants: the lane's B record (dead MMA columns 3..7 reuse plane 0 and get weight 0)
// and the digit weights of its two D columns n0 = 2tig, n1 = 2tig + 1.
struct PLane {
  uint32_t boff;
  float w0, w1;
  int tig;
};
__device__ __forceinline__ PLane p_lane(int lane) {
  const int grp = lane >> 2, tig = lane & 3, dg = grp < 3 ? grp : 0;
  PLane L;
  L.boff = (uint32_t)(dg * 4 + tig) * 80;
  L.w0 = tig == 0 ? 1.f : tig == 1 ? 1.f / 64516.f : 0.f;
  L.w1 = tig == 0 ? 1.f / 254.f : 0.f;
  L.tig = tig;
  return L;
}

// Digitise the phase input (RMS-normalised when nw is set) with one round of loads: warp w
// holds super-blocks w, w+14, ... in registers, lane l the eight values 8(l&3)..8(l&3)+7 of
// 32-block l>>2, and the norm's sum of squares comes from the same registers. x ~= s * (a + b/254 +
// c/254^2), s = max|x|/127 per super-block (the same digits as the stand-alone GEMV). The block
// maximum is one warp reduction over the bit patterns (non-negative floats order as integers), the
// digit bytes are packed from the bit patterns of the rounding additions, and a 32-block's digit
// sums meet over the four lanes that hold it (a 16-run's over two).
// SM: x is a row in this CTA's shared memory (the tensor-parallel sum, p_sum_parts), else in global
// memory (read through L2).
__device__ __forceinline__ void digits254_bits(float t, uint32_t &a, uint32_t &b, uint32_t &c) {
  // digits254 without the final masks: each digit is the low byte of the returned bit pattern
  const float M = 12582912.f;
  const float ta = __fadd_rn(t, M), r1 = __fmul_rn(__fsub_rn(t, __fsub_rn(ta, M)), 254.f);
  const float tb = __fadd_rn(r1, M), r2 = __fmul_rn(__fsub_rn(r1, __fsub_rn(tb, M)), 254.f);
  const float tc = __fadd_rn(r2, M);
  a = __float_as_uint(ta);
  b = __float_as_uint(tb);
  c = __float_as_uint(tc);
}
// the low bytes of w0..w3 as one word (byte e from w_e)
__device__ __forceinline__ uint32_t pack_low_bytes(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3) {
  return __byte_perm(__byte_perm(w0, w1, 0x0040), __byte_perm(w2, w3, 0x0040), 0x5410);
}

template <bool SM>
__device__ void p_digitise(const float *x, const float *nw, float eps, int cols, bool q6, const PX &X, float *red, int *sums,
                           int warp, int lane) {
  const int nsb = cols >> 8;
  const int j = lane >> 2, q = lane & 3;  // 32-block, quarter (eight values k = 8q..8q+7)
  float4 v[P_MAXSBW][2];
#pragma unroll
  for (int i = 0; i < P_MAXSBW; i++) {
    const int sb = warp + P_CWARPS * i;
    const int col = 256 * sb + 32 * j + 8 * q;
    const bool in = sb < nsb;
#pragma unroll
    for (int h = 0; h < 2; h++) {
      if (SM) v[i][h] = in ? *reinterpret_cast<const float4 *>(x + col + 4 * h) : make_float4(0.f, 0.f, 0.f, 0.f);
      else v[i][h] = in ? __ldcg(reinterpret_cast<const float4 *>(x + col + 4 * h)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    // the norm weights are read after the block-wide sum: bring them into L1 now
    if (in && nw) asm volatile("prefetch.global.L1 [%0];" ::"l"(nw + col));
  }
  if (nw) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < P_MAXSBW; i++)
#pragma unroll
      for (int h = 0; h < 2; h++)
        ss = fmaf(v[i][h].x, v[i][h].x, fmaf(v[i][h].y, v[i][h].y, fmaf(v[i][h].z, v[i][h].z, fmaf(v[i][h].w, v[i][h].w, ss))));
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    bar_comp();
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < P_CWARPS; w++) t += red[w];
    const float inv = rsqrtf(t / (float)cols + eps);
#pragma unroll
    for (int i = 0; i < P_MAXSBW; i++) {
      const int sb = warp + P_CWARPS * i;
      if (sb >= nsb) continue;
      const int col = 256 * sb + 32 * j + 8 * q;
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const float4 w = __ldg(reinterpret_cast<const float4 *>(nw + col + 4 * h));
        v[i][h] = make_float4(v[i][h].x * inv * w.x, v[i][h].y * inv * w.y, v[i][h].z * inv * w.z, v[i][h].w * inv * w.w);
      }
    }
  }
  // record words of this lane: plane dg, k = 8q..8q+3 at tig 2(q&1), k = 8q+4.. at tig 2(q&1)+1,
  // half hi = q >> 1 (k >= 16), 32-block j
  const int tg0 = 2 * (q & 1), hi = q >> 1;
#pragma unroll
  for (int i = 0; i < P_MAXSBW; i++) {
    const int sb = warp + P_CWARPS * i;
    if (sb >= nsb) continue;
    float m = fmaxf(fmaxf(fmaxf(fabsf(v[i][0].x), fabsf(v[i][0].y)), fmaxf(fabsf(v[i][0].z), fabsf(v[i][0].w))),
                    fmaxf(fmaxf(fabsf(v[i][1].x), fabsf(v[i][1].y)), fmaxf(fabsf(v[i][1].z), fabsf(v[i][1].w))));
    const float amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(m)));
    // digit scale: the fast reciprocal is within 2 ulp of 127 / amax, which only moves the
    // digits by that much relative to the exact scale sxs they are multiplied back with
    const float sc = amax > 0.f ? __fdividef(127.f, amax) : 0.f;
    if (lane == 0) X.sxs[sb] = amax > 0.f ? amax / 127.f : 0.f;
    uint32_t wa[3][2];  // [plane][word]
#pragma unroll
    for (int h = 0; h < 2; h++) {
      uint32_t a0, b0, c0, a1, b1, c1, a2, b2, c2, a3, b3, c3;
      digits254_bits(v[i][h].x * sc, a0, b0, c0);
      digits254_bits(v[i][h].y * sc, a1, b1, c1);
      digits254_bits(v[i][h].z * sc, a2, b2, c2);
      digits254_bits(v[i][h].w * sc, a3, b3, c3);
      wa[0][h] = pack_low_bytes(a0, a1, a2, a3);
      wa[1][h] = pack_low_bytes(b0, b1, b2, b3);
      wa[2][h] = pack_low_bytes(c0, c1, c2, c3);
    }
    uint8_t *rec = X.brec + (size_t)sb * 960 + j * 8 + hi * 4;
#pragma unroll
    for (int dg = 0; dg < 3; dg++) {
      *reinterpret_cast<uint32_t *>(rec + (dg * 4 + tg0) * 80) = wa[dg][0];
      *reinterpret_cast<uint32_t *>(rec + (dg * 4 + tg0 + 1) * 80) = wa[dg][1];
      int s = __dp4a((int)wa[dg][0], 0x01010101, __dp4a((int)wa[dg][1], 0x01010101, 0));
      s += __shfl_xor_sync(0xffffffffu, s, 1);  // 16-run 2j + hi
      if (q6) {
        if ((q & 1) == 0) sums[dg * 16 + 2 * j + hi] = s;
      } else {
        s += __shfl_xor_sync(0xffffffffu, s, 2);  // 32-block j
        if (q == 0) sums[dg * 16 + j] = s;
      }
    }
    __syncwarp();
    // lane (grp = dg, tig) of the digit-sum MMA holds the sums k = 4tig..4tig+3 of column dg,
    // split into low bytes (unsigned) and high bytes (signed): sum = 256*hi + lo
    {
      const int grp = lane >> 2, tig = lane & 3;
      uint32_t lo = 0u, hw = 0u;
      if (grp < 3 && (q6 || tig < 2)) {
#pragma unroll
        for (int m2 = 0; m2 < 4; m2++) {
          const int sv = sums[grp * 16 + 4 * tig + m2];
          lo |= ((uint32_t)sv & 255u) << (8 * m2);
          hw |= ((uint32_t)(sv >> 8) & 255u) << (8 * m2);
        }
      }
      *reinterpret_cast<uint2 *>(X.dsw + (size_t)sb * 256 + lane * 8) = make_uint2(lo, hw);
    }
    __syncwarp();
  }
}

// Tensor parallelism: the phase input is x plus the nparts partial rows at part (stride floats
// apart), added in rank order (the same sum on every CTA of every rank) into the shared-memory row
// dst; CTA (super-block mod grid) also stores its super-blocks of the sum to x_out, the residual
// stream that later phases read. Compute warps only; ends with their named barrier.
__device__ void p_sum_parts(const float *x, const float *part, int nparts, int stride, int cols, float *dst, float *x_out) {
  const int tid = threadIdx.x;
  for (int c4 = tid; c4 < (cols >> 2); c4 += P_CWARPS * 32) {
    const int col = 4 * c4;
    float4 v = __ldcg(reinterpret_cast<const float4 *>(x + col));
    // the partial rows requested together (at most P_TP_MAX), then added in rank order
    float4 w[P_TP_MAX];
#pragma unroll
    for (int j = 0; j < P_TP_MAX; j++)
      w[j] = j < nparts ? __ldcg(reinterpret_cast<const float4 *>(part + (size_t)j * stride + col)) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < P_TP_MAX; j++)
      if (j < nparts) v = make_float4(v.x + w[j].x, v.y + w[j].y, v.z + w[j].z, v.w + w[j].w);
    *reinterpret_cast<float4 *>(dst + col) = v;
    if (x_out && (col >> 8) % (int)gridDim.x == (int)blockIdx.x) __stcg(reinterpret_cast<float4 *>(x_out + col), v);
  }
  asm volatile("bar.sync 3, %0;" ::"n"(P_CWARPS * 32) : "memory");
}

// MMA shapes with the operand signedness the chunk math needs (D = A*B, zero C).
__device__ __forceinline__ void mma_k32_uu(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(0u), "r"(0u), "r"(b0), "r"(0u), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void mma_k32_us(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(0u), "r"(0u), "r"(b0), "r"(0u), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void mma_k16_su(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm("mma.sync.aligned.m16n8k16.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%8,%9,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(b0), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void mma_k16_ss(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%8,%9,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(b0), "r"(0), "r"(0), "r"(0), "r"(0));
}

// One Q4_K tile chunk (16 rows x 256 columns, staged in shared memory at c) against the
// digit records of super-block kb:
//   sum_j (d*sc_j*q - dmin*mn_j) x = s*(d*sum_j sc_j*D_j - dmin*sum_j mn_j*Sdig_j)
// The high nibbles enter the MMA as 16*q (byte & 0xF0, still a u8 operand) and are summed
// separately, then divided by 16 exactly. sum_j mn_j*Sdig_j is itself one small MMA: the six
// packed 6-bit mins of each row are the A fragment (k = j), the digit sums (split into a low and
// a high byte) the B fragment.
__device__ __forceinline__ void p_q4k(const uint8_t *c, int kb, const PX &X, const PLane &P, int lane, float (&acc)[2]) {
  Q4KRegs r;
#pragma unroll
  for (int g = 0; g < 4; g++) r.qs[g] = *reinterpret_cast<const uint4 *>(c + 512 * g + 16 * lane);
  const int grp = lane >> 2, tig = lane & 3;
  r.h0 = *reinterpret_cast<const uint4 *>(c + 2048 + 16 * grp);
  r.h1 = *reinterpret_cast<const uint4 *>(c + 2048 + 16 * (grp + 8));
  const uint32_t M4 = 0x0F0F0F0Fu, H4 = 0xF0F0F0F0u;
  const uint32_t sc_lo0 = r.h0.y & 0x3F3F3F3Fu, mn_lo0 = r.h0.z & 0x3F3F3F3Fu;
  const uint32_t sc_hi0 = (r.h0.w & M4) | ((r.h0.y >> 2) & 0x30303030u);
  const uint32_t mn_hi0 = ((r.h0.w >> 4) & M4) | ((r.h0.z >> 2) & 0x30303030u);
  const uint32_t sc_lo1 = r.h1.y & 0x3F3F3F3Fu, mn_lo1 = r.h1.z & 0x3F3F3F3Fu;
  const uint32_t sc_hi1 = (r.h1.w & M4) | ((r.h1.y >> 2) & 0x30303030u);
  const uint32_t mn_hi1 = ((r.h1.w >> 4) & M4) | ((r.h1.z >> 2) & 0x30303030u);
  const uint4 *bp = reinterpret_cast<const uint4 *>(X.brec + (size_t)kb * 960 + P.boff);
  uint4 B[4];
#pragma unroll
  for (int i = 0; i < 4; i++) B[i] = bp[i];
  const uint2 dw = *reinterpret_cast<const uint2 *>(X.dsw + (size_t)kb * 256 + lane * 8);
  // mins term: A = mins of rows grp / grp+8 at k = j (tig 0: j 0..3, tig 1: j 4..7)
  const uint32_t am0 = tig == 0 ? mn_lo0 : tig == 1 ? mn_hi0 : 0u, am1 = tig == 0 ? mn_lo1 : tig == 1 ? mn_hi1 : 0u;
  int Ml[4], Mh[4];
  mma_k32_uu(Ml, am0, am1, dw.x);
  mma_k32_us(Mh, am0, am1, dw.y);
  // |D| <= 32*15*127 = 60960 (low) / 16x that (high); x sc <= 63, 4 sub-blocks each: < 2.5e8.
  int E00 = 0, E01 = 0, E10 = 0, E11 = 0, O00 = 0, O01 = 0, O10 = 0, O11 = 0;
#pragma unroll
  for (int g = 0; g < 4; g++) {
    const uint32_t w[4] = {r.qs[g].x, r.qs[g].y, r.qs[g].z, r.qs[g].w};
#pragma unroll
    for (int half = 0; half < 2; half++) {
      const int s = 2 * g + half;
      const uint32_t m = half ? H4 : M4;
      const uint32_t aa[4] = {w[0] & m, w[1] & m, w[2] & m, w[3] & m};
      const int sc0 = ubyte(s < 4 ? sc_lo0 : sc_hi0, s & 3), sc1 = ubyte(s < 4 ? sc_lo1 : sc_hi1, s & 3);
      const uint4 bq = B[s >> 1];
      int D[4];
      mma_k32(D, aa, (s & 1) ? bq.z : bq.x, (s & 1) ? bq.w : bq.y);
      if (half) {
        O00 += sc0 * D[0];
        O01 += sc0 * D[1];
        O10 += sc1 * D[2];
        O11 += sc1 * D[3];
      } else {
        E00 += sc0 * D[0];
        E01 += sc0 * D[1];
        E10 += sc1 * D[2];
        E11 += sc1 * D[3];
      }
    }
  }
  const int I00 = E00 + (O00 >> 4), I01 = E01 + (O01 >> 4), I10 = E10 + (O10 >> 4), I11 = E11 + (O11 >> 4);
  const int M00 = Ml[0] + (Mh[0] << 8), M01 = Ml[1] + (Mh[1] << 8), M10 = Ml[2] + (Mh[2] << 8), M11 = Ml[3] + (Mh[3] << 8);
  const float d0 = h2f(r.h0.x), d1 = h2f(r.h1.x), m0 = h2f(r.h0.x >> 16), m1 = h2f(r.h1.x >> 16);
  const float sx = X.sxs[kb];
  acc[0] = fmaf(sx, fmaf(P.w0, d0 * (float)I00 - m0 * (float)M00, P.w1 * (d0 * (float)I01 - m0 * (float)M01)), acc[0]);
  acc[1] = fmaf(sx, fmaf(P.w0, d1 * (float)I10 - m1 * (float)M10, P.w1 * (d1 * (float)I11 - m1 * (float)M11)), acc[1]);
}

// One Q6_K tile chunk: sum_j d*sc_j*(q-32) x = s*d*(sum_j sc_j*D_j - 32*sum_j sc_j*Sdig_j), the
// second sum one k16 MMA whose A fragment is the row's raw int8 scale words (k = 16-run j).
__device__ __forceinline__ void p_q6k(const uint8_t *c, int kb, const PX &X, const PLane &P, int lane, float (&acc)[2]) {
  Q6KRegs r;
#pragma unroll
  for (int k = 0; k < 4; k++) r.ql[k] = *reinterpret_cast<const uint4 *>(c + 512 * k + 16 * lane);
  r.qh[0] = *reinterpret_cast<const uint4 *>(c + 2048 + 16 * lane);
  r.qh[1] = *reinterpret_cast<const uint4 *>(c + 2560 + 16 * lane);
  const int grp = lane >> 2, tig = lane & 3;
  r.s0 = *reinterpret_cast<const uint4 *>(c + 3072 + 16 * grp);
  r.s1 = *reinterpret_cast<const uint4 *>(c + 3072 + 16 * (grp + 8));
  r.d = (uint32_t)*reinterpret_cast<const uint16_t *>(c + 3328 + 2 * grp) |
        ((uint32_t)*reinterpret_cast<const uint16_t *>(c + 3328 + 2 * (grp + 8)) << 16);
  const uint32_t M4 = 0x0F0F0F0Fu, T3 = 0x03030303u;
  const uint32_t sw0[4] = {r.s0.x, r.s0.y, r.s0.z, r.s0.w}, sw1[4] = {r.s1.x, r.s1.y, r.s1.z, r.s1.w};
  const uint4 *bp = reinterpret_cast<const uint4 *>(X.brec + (size_t)kb * 960 + P.boff);
  uint4 B[4];
#pragma unroll
  for (int i = 0; i < 4; i++) B[i] = bp[i];
  const uint2 dw = *reinterpret_cast<const uint2 *>(X.dsw + (size_t)kb * 256 + lane * 8);
  // offset term: A = the 16 int8 scales of rows grp / grp+8 (k = 16-run), this lane's 4 of them
  const uint32_t as0 = tig == 0 ? sw0[0] : tig == 1 ? sw0[1] : tig == 2 ? sw0[2] : sw0[3];
  const uint32_t as1 = tig == 0 ? sw1[0] : tig == 1 ? sw1[1] : tig == 2 ? sw1[2] : sw1[3];
  int Tl[4], Th[4];
  mma_k16_su(Tl, as0, as1, dw.x);
  mma_k16_ss(Th, as0, as1, dw.y);
  int I00 = 0, I01 = 0, I10 = 0, I11 = 0;
#pragma unroll
  for (int seg = 0; seg < 2; seg++) {
    const uint32_t hw[4] = {r.qh[seg].x, r.qh[seg].y, r.qh[seg].z, r.qh[seg].w};
#pragma unroll
    for (int quarter = 0; quarter < 4; quarter++) {
      const int qp = quarter & 1, nib = quarter >> 1;
      const uint4 lw = r.ql[2 * seg + qp];
      const uint32_t l[4] = {lw.x, lw.y, lw.z, lw.w};
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int s = 8 * seg + 2 * quarter + h;  // sub-block of 16 values; 32-block s/2, half h
        const uint32_t a0 = ((l[2 * h] >> (4 * nib)) & M4) | (((hw[2 * h] >> (2 * quarter)) & T3) << 4);
        const uint32_t a1 = ((l[2 * h + 1] >> (4 * nib)) & M4) | (((hw[2 * h + 1] >> (2 * quarter)) & T3) << 4);
        const int sc0 = sbyte(sw0[s >> 2], s & 3), sc1 = sbyte(sw1[s >> 2], s & 3);
        const uint4 bq = B[s >> 2];
        const int j = s >> 1;
        const uint32_t b0 = (j & 1) ? (h ? bq.w : bq.z) : (h ? bq.y : bq.x);
        int D[4];
        mma_k16(D, a0, a1, b0);
        // |D| <= 16*63*127 = 128016; x |sc| <= 128 and 16 sub-blocks: < 2.7e8.
        I00 += sc0 * D[0];
        I01 += sc0 * D[1];
        I10 += sc1 * D[2];
        I11 += sc1 * D[3];
      }
    }
  }
  // |T| <= 16*128*2032 = 4.2e6 per entry; 32*T well inside int32
  I00 -= 32 * (Tl[0] + (Th[0] << 8));
  I01 -= 32 * (Tl[1] + (Th[1] << 8));
  I10 -= 32 * (Tl[2] + (Th[2] << 8));
  I11 -= 32 * (Tl[3] + (Th[3] << 8));
  const float d0 = h2f(r.d), d1 = h2f(r.d >> 16);
  const float sx = X.sxs[kb];
  acc[0] = fmaf(sx, fmaf(P.w0, d0 * (float)I00, P.w1 * (d0 * (float)I01)), acc[0]);
  acc[1] = fmaf(sx, fmaf(P.w0, d1 * (float)I10, P.w1 * (d1 * (float)I11)), acc[1]);
}

struct GemvCtx {
  const PGemv *g;
  const PersistArgs *a;
  float best_v;  // greedy tracking (per lane)
  int best_i;
  int row0;      // global index of output row 0 (the vocabulary offset of this rank's LM head rows)
  // residual-add epilogues: this lane's rows of the CTA's first P_PRE tiles, loaded at phase start
  int pre_t0;
  float pre[4];
};
constexpr int P_PRE = 4;

// Epilogue of one finished tile: lane r < 16 holds the value of tile row r.
__device__ __forceinline__ void p_epilogue(GemvCtx &C, int t, float v, int lane) {
  const PGemv &g = *C.g;
  if (g.epi == EPI_GLU_SILU || g.epi == EPI_GLU_GELU) {
    const float up = __shfl_sync(0xffffffffu, v, (lane + 8) & 31);
    if (lane < 8 && t * 16 + lane < g.rows) g.y[t * 8 + lane] = (g.epi == EPI_GLU_SILU ? g2_silu(v) : g2_gelu(v)) * up;
    return;
  }
  const int row = t * 16 + lane;
  if (lane < 16 && row < g.rows) {
    float val = v;
    if (g.bias) val += __ldg(g.bias + row);
    if (g.push) {
      // this rank's partial row into its slot of every rank's exchange buffer (peer stores over NVLink)
      const PersistArgs &a = *C.a;
      const size_t off = ((size_t)(g.push - 1) * P_TP_MAX + a.rank) * a.hidden + row;
      for (int j = 0; j < a.tp; j++) reinterpret_cast<float *>(a.xbuf[j] + a.x_slot)[off] = val;
      return;
    }
    if (g.epi == EPI_ADD) {
      const int k = t - C.pre_t0;
      const float old = k == 0 ? C.pre[0] : k == 1 ? C.pre[1] : k == 2 ? C.pre[2] : k == 3 ? C.pre[3] : __ldcg(g.y + row);
      val = old + val;
      g.y[row] = val;
    } else if (g.epi == EPI_SILU) {
      val = g2_silu(val);
      g.y[row] = val;
    } else {
      g.y[row] = val;
    }
    if (g.argmax && isfinite(val) && better(val, C.row0 + row, C.best_v, C.best_i)) {
      C.best_v = val;
      C.best_i = C.row0 + row;
    }
  }
}

// ------------------------------------------------------------------ attention item

// One (kv head, key split) of decode attention by consumer warps 0..AW-1 (named barrier 2);
// same math and merge order as attention_kernel.
// Shared memory of one attention item (floats): [K|V stage 1][K|V stage 0][q][new k][new v],
// a stage holding 32 rows of hd + 4 floats each for K and V.
__device__ __forceinline__ int attn_stage_floats(int hd) { return 2 * 32 * (hd + 4); }
__device__ __forceinline__ float *attn_stage(float *sm, int hd, int st) { return sm + (st ? 0 : attn_stage_floats(hd)); }

// Issue the cp.async copies of K/V rows [tile, min(tile + 32, p1)) of kv head kh into stage st
// (the row of the position being decoded comes from shared memory instead) and commit them.
// Warps 0..nw-1 issue them (tid < 32 * nw).
__device__ void p_attn_stage(const PAttn &A, int pos, int kh, int p1, int tile, float *sm, int st, int tid, int nw) {
  const int hd = A.hd, RS = hd + 4, end = pos + 1;
  const bool owns_new = p1 == end;
  const float *kb = A.k + (int64_t)kh * A.capacity * hd, *vb = A.v + (int64_t)kh * A.capacity * hd;
  const int cnt = min(32, p1 - tile);
  float *ks = attn_stage(sm, hd, st), *vs = ks + 32 * RS;
  // a warp per key row (the ring slot computed once per row), lanes over its 16-byte pieces
  const int w = tid >> 5, lane = tid & 31;
  for (int r = w; r < cnt; r += nw) {
    const int p = tile + r;
    if (owns_new && p == end - 1) continue;
    const int64_t row = (int64_t)(p % A.capacity) * hd;
    for (int c = 4 * lane; c < hd; c += 128) {
      cp_async16(ks + r * RS + c, kb + row + c);
      cp_async16(vs + r * RS + c, vb + row + c);
    }
  }
  cp_commit();
}

// Key split of the item: positions [p0, p1).
__device__ __forceinline__ void attn_split(const PAttn &A, int pos, int nspmax, int &chunk, int &nsp) {
  const int end = pos + 1, L = end < A.window ? end : A.window;
  chunk = (L + nspmax - 1) / nspmax;
  if (chunk < 32) chunk = 32;
  nsp = (L + chunk - 1) / chunk;
}

// One (kv head, key split) of decode attention. Every compute warp enters; warps 0..AW-1 (named
// barrier 2; AW = 8 when head_dim is a multiple of 32, else 4) stage K/V, rotate q/k and run the
// tiles, and all 14 merge the key splits of the kv head when this CTA is the last to finish one (named
// barrier 3). Per 32-key tile:
//   scores   warp w sums dims [w*hd/AW, (w+1)*hd/AW) for every query head of the group, lane = key
//            (each K row is read once for all heads), the AW parts added in warp order;
//   softmax  warp w owns heads w, w+AW: running max / sum per head (shared memory), the tile's
//            probabilities to shared memory;
//   P.V      warp w takes keys j = w (mod AW), lane = four dims, every head at once (each V row read
//            once), its partial sums rescaled by the heads' corrections; the AW warps' sums are
//            added in warp order at the end.
// `staged`: stage 0 already holds the first K/V tile (issued while the QKV projection ran).
constexpr int AW_MAX = 8;  // most warps of the tile work (the score scratch is sized for it)
__device__ __forceinline__ float *attn_scratch(float *sm, int G, int hd) { return sm + 2 * attn_stage_floats(hd) + G * hd + 2 * hd; }

template <int AW>
__device__ __forceinline__ void abar() { asm volatile("bar.sync 2, %0;" ::"n"(AW * 32) : "memory"); }

template <int AW>
__device__ void p_attn_item(const PAttn &A, int pos, int kh, int sp, int nsp, int chunk, int nspmax, float *sm, float *att_part,
                            unsigned *att_ctr, int *last_s, bool staged, int tr_step, int tr_phase) {
  (void)tr_step;
  (void)tr_phase;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = A.heads / A.kv_heads, hd = A.hd, hd4 = hd >> 2, RS = hd + 4;
  float *q_s = sm + 2 * attn_stage_floats(hd), *kn_s = q_s + G * hd, *vn_s = kn_s + hd;
  float *sc_s = attn_scratch(sm, G, hd);  // [AW][8][32] score parts
  float *pr_s = sc_s + AW * 8 * 32;       // [32][8] probabilities of the tile
  float *st_s = pr_s + 32 * 8;            // [3][8] running max, running sum, correction
  const int end = pos + 1, begin = end - (end < A.window ? end : A.window);
  const int p0 = begin + sp * chunk, p1 = min(end, p0 + chunk);
  const bool owns_new = p1 == end;
  const int ntiles = (p1 - p0 + 31) / 32;
  const int PR = hd + 4;
  float *out_base = A.out + (int64_t)kh * G * hd;
  if (warp < AW) {
    if (!staged) p_attn_stage(A, pos, kh, p1, p0, sm, 0, tid, AW);
    if (ntiles > 1) p_attn_stage(A, pos, kh, p1, p0 + 32, sm, 1, tid, AW);
    const int hq = G + (owns_new ? 1 : 0);
    // this lane's RoPE (cos, sin) pairs, requested together with q/k/v (the same for every head)
    const int half = A.rot / 2;
    const float2 *tb = A.table + (int64_t)pos * half;
    float2 cs[4];
#pragma unroll
    for (int k = 0; k < 4; k++) cs[k] = lane + 32 * k < half ? __ldg(tb + lane + 32 * k) : make_float2(1.f, 0.f);
    for (int i = tid; i < hq * hd; i += AW * 32) {
      const int g = i / hd, d = i - g * hd;
      const float *src = g < G ? A.qkv + (int64_t)(kh * G + g) * hd : A.qkv + (int64_t)(A.heads + kh) * hd;
      (g < G ? q_s + g * hd : kn_s)[d] = __ldcg(src + d);
    }
    if (owns_new)
      for (int d = tid; d < hd; d += AW * 32) vn_s[d] = __ldcg(A.qkv + (int64_t)(A.heads + A.kv_heads + kh) * hd + d);
    if (tid < 8) {
      st_s[tid] = -FLT_MAX;
      st_s[8 + tid] = 0.f;
    }
    abar<AW>();
    for (int g = warp; g < hq; g += AW) {
      float *hv = g < G ? q_s + g * hd : kn_s;
      const float *nw = g < G ? A.q_norm : A.k_norm;
      if (nw) {
        float ss = 0.f;
        for (int d = lane; d < hd; d += 32) ss = fmaf(hv[d], hv[d], ss);
        const float inv = rsqrtf(warp_sum(ss) / (float)hd + A.eps);
        __syncwarp();
        for (int d = lane; d < hd; d += 32) hv[d] = hv[d] * inv * nw[d];
        __syncwarp();
      }
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const int i = lane + 32 * k;
        if (i >= half) break;
        const int ia = A.mode == 0 ? i : 2 * i, ib = A.mode == 0 ? i + half : 2 * i + 1;
        const float l = hv[ia], r = hv[ib];
        hv[ia] = l * cs[k].x - r * cs[k].y;
        hv[ib] = l * cs[k].y + r * cs[k].x;
      }
      __syncwarp();
    }
    abar<AW>();
    if (tid == 0) P_TRACE(tr_step, tr_phase, 1);
    if (owns_new) {
      const int slot = pos % A.capacity;
      float *kd = A.k + ((int64_t)kh * A.capacity + slot) * hd, *vd = A.v + ((int64_t)kh * A.capacity + slot) * hd;
      for (int d = tid; d < hd; d += AW * 32) { kd[d] = kn_s[d]; vd[d] = vn_s[d]; }
    }
    const int dq = hd / (4 * AW);  // float4s of the score dims of one warp
    float4 acc[8];
#pragma unroll
    for (int g = 0; g < 8; g++) acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int ti = 0; ti < ntiles; ti++) {
      const int tile = p0 + ti * 32, cnt = min(32, p1 - tile), st = ti & 1;
      if (ti + 1 < ntiles) cp_wait<1>(); else cp_wait<0>();
      abar<AW>();
      float *ks = attn_stage(sm, hd, st), *vs = ks + 32 * RS;
      if (owns_new && tile + cnt == end) {
        const int r = end - 1 - tile;
        for (int d = tid; d < hd; d += AW * 32) { ks[r * RS + d] = kn_s[d]; vs[r * RS + d] = vn_s[d]; }
        abar<AW>();
      }
      {  // scores: this warp's quarter of the dims, every head, lane = key
        const float4 *kr = reinterpret_cast<const float4 *>(ks + lane * RS) + warp * dq;
        float sp2[8][2];
#pragma unroll
        for (int g = 0; g < 8; g++) sp2[g][0] = sp2[g][1] = 0.f;
        for (int i = 0; i < dq; i++) {
          const float4 k4 = kr[i];
#pragma unroll
          for (int g = 0; g < 8; g++) {
            if (g < G) {
              const float4 q = reinterpret_cast<const float4 *>(q_s + g * hd)[warp * dq + i];
              sp2[g][0] = fmaf(q.x, k4.x, fmaf(q.y, k4.y, sp2[g][0]));
              sp2[g][1] = fmaf(q.z, k4.z, fmaf(q.w, k4.w, sp2[g][1]));
            }
          }
        }
#pragma unroll
        for (int g = 0; g < 8; g++)
          if (g < G) sc_s[(warp * 8 + g) * 32 + lane] = sp2[g][0] + sp2[g][1];
      }
      abar<AW>();
      for (int g = warp; g < G; g += AW) {  // online softmax of head g over this tile
        float sv = sc_s[g * 32 + lane];
#pragma unroll
        for (int w = 1; w < AW; w++) sv += sc_s[(w * 8 + g) * 32 + lane];
        const bool live = lane < cnt;
        sv = live ? sv * A.scale : -FLT_MAX;
        const float mo = st_s[g], mn = fmaxf(mo, warp_max(sv)), corr = expf(mo - mn);
        const float e = live ? expf(sv - mn) : 0.f;
        const float ls = warp_sum(e);
        pr_s[lane * 8 + g] = e;
        if (lane == 0) {
          st_s[g] = mn;
          st_s[8 + g] = fmaf(st_s[8 + g], corr, ls);
          st_s[16 + g] = corr;
        }
      }
      abar<AW>();
      if (lane < hd4) {  // P.V: keys j = warp (mod AW), four dims per lane, every head
        float cr[8];
#pragma unroll
        for (int g = 0; g < 8; g++) cr[g] = g < G ? st_s[16 + g] : 0.f;
#pragma unroll
        for (int g = 0; g < 8; g++) acc[g] = make_float4(acc[g].x * cr[g], acc[g].y * cr[g], acc[g].z * cr[g], acc[g].w * cr[g]);
        for (int j = warp; j < cnt; j += AW) {
          const float4 v = reinterpret_cast<const float4 *>(vs + j * RS)[lane];
          const float4 pa = reinterpret_cast<const float4 *>(pr_s + j * 8)[0], pb = reinterpret_cast<const float4 *>(pr_s + j * 8)[1];
          const float pw[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
#pragma unroll
          for (int g = 0; g < 8; g++)
            if (g < G)
              acc[g] = make_float4(fmaf(pw[g], v.x, acc[g].x), fmaf(pw[g], v.y, acc[g].y), fmaf(pw[g], v.z, acc[g].z),
                                   fmaf(pw[g], v.w, acc[g].w));
        }
      }
      abar<AW>();
      if (ti + 2 < ntiles) p_attn_stage(A, pos, kh, p1, tile + 64, sm, st, tid, AW);
    }
    if (tid == 0) P_TRACE(tr_step, tr_phase, 2);
    // the AW warps' P.V sums, added in warp order (stage 1 is free now: no copy is in flight)
    float4 *cb = reinterpret_cast<float4 *>(sm);  // [AW][G][hd4]
    if (lane < hd4) {
#pragma unroll
      for (int g = 0; g < 8; g++)
        if (g < G) cb[(warp * G + g) * hd4 + lane] = acc[g];
    }
    abar<AW>();
    for (int i = tid; i < G * hd4; i += AW * 32) {
      const int g = i / hd4, d4 = i - g * hd4;
      float4 t = cb[g * hd4 + d4];
#pragma unroll
      for (int w = 1; w < AW; w++) {
        const float4 u = cb[(w * G + g) * hd4 + d4];
        t = make_float4(t.x + u.x, t.y + u.y, t.z + u.z, t.w + u.w);
      }
      if (nsp == 1) {
        const float l = st_s[8 + g];
        reinterpret_cast<float4 *>(out_base + g * hd)[d4] = make_float4(t.x / l, t.y / l, t.z / l, t.w / l);
      } else {
        float *part = att_part + ((int64_t)kh * nspmax + sp) * G * PR;
        __stcg(reinterpret_cast<float4 *>(part + g * PR) + d4, t);
        if (d4 == 0) {
          __stcg(part + g * PR + hd, st_s[g]);
          __stcg(part + g * PR + hd + 1, st_s[8 + g]);
        }
      }
    }
    if (nsp > 1) __threadfence();
    abar<AW>();
    if (tid == 0 && nsp > 1) *last_s = atomicAdd(att_ctr + kh, 1u) == (unsigned)(nsp - 1);
    if (tid == 0) P_TRACE(tr_step, tr_phase, 4);
  }
  if (nsp == 1) return;
  bar_comp();  // every compute warp learns whether this CTA merges the kv head's splits
  if (!*last_s) return;
  __threadfence();
  // merge of the nsp splits by the 14 compute warps: warp g < G turns head g's (max, sum) pairs
  // into weights; then (output float4, split group) items sum their splits' partials
  const float *pb = att_part + (int64_t)kh * nspmax * G * PR;
  const int64_t sstride = (int64_t)G * PR;
  float *wt_s = attn_scratch(sm, G, hd);  // [8][64] weights (the score scratch is free now)
  if (warp < G) {
    const float *ph = pb + warp * PR;
    const float ma = lane < nsp ? __ldcg(ph + lane * sstride + hd) : -FLT_MAX;
    const float mb = lane + 32 < nsp ? __ldcg(ph + (lane + 32) * sstride + hd) : -FLT_MAX;
    const float la = lane < nsp ? __ldcg(ph + lane * sstride + hd + 1) : 0.f;
    const float lb = lane + 32 < nsp ? __ldcg(ph + (lane + 32) * sstride + hd + 1) : 0.f;
    const float M = warp_max(fmaxf(ma, mb));
    const float wa = lane < nsp ? expf(ma - M) : 0.f, wb = lane + 32 < nsp ? expf(mb - M) : 0.f;
    const float den = warp_sum(fmaf(wa, la, wb * lb));
    wt_s[warp * 64 + lane] = wa / den;
    wt_s[warp * 64 + lane + 32] = wb / den;
  }
  bar_comp();
  const int W4 = G * hd4, NG = max(1, min(8, (P_CWARPS * 32) / W4));
  float4 *cb = reinterpret_cast<float4 *>(sm);  // [NG][W4] group sums
  if (tid < NG * W4) {
    const int item = tid % W4, grp = tid / W4, g = item / hd4, d4 = item - g * hd4;
    const float *ph = pb + g * PR;
    float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j0 = grp; j0 < nsp; j0 += 8 * NG) {
      float4 pv[8];
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const int j = j0 + u * NG;
        pv[u] = j < nsp ? __ldcg(reinterpret_cast<const float4 *>(ph + j * sstride) + d4) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const int j = j0 + u * NG;
        const float w = j < nsp ? wt_s[g * 64 + j] : 0.f;
        num = make_float4(fmaf(w, pv[u].x, num.x), fmaf(w, pv[u].y, num.y), fmaf(w, pv[u].z, num.z), fmaf(w, pv[u].w, num.w));
      }
    }
    cb[grp * W4 + item] = num;
  }
  bar_comp();
  for (int i = tid; i < W4; i += P_CWARPS * 32) {
    const int g = i / hd4, d4 = i - g * hd4;
    float4 t = cb[i];
    for (int q = 1; q < NG; q++) {
      const float4 u = cb[q * W4 + i];
      t = make_float4(t.x + u.x, t.y + u.y, t.z + u.z, t.w + u.w);
    }
    reinterpret_cast<float4 *>(out_base + g * hd)[d4] = t;
  }
  if (tid == 0) att_ctr[kh] = 0u;
  if (tid == 0) P_TRACE(tr_step, tr_phase, 5);
}

// ------------------------------------------------------------------ embedding

template <int T>
__device__ __forceinline__ float p_embed_elem(const PersistArgs &a, int token, int col) {
  if (a.embd_tiled) {
    if constexpr (T == Q4_K || T == Q6_K) return dequant_tiled<T>(a.embd, a.hidden / 256, token, col);
    return 0.f;
  }
  return dequant_elem<T>(a.embd + (int64_t)token * a.embd_drow, a.hidden / block_elems_dev<T>(), col);
}
__device__ float p_embed_value(const PersistArgs &a, int token, int col) {
  switch (a.embd_type) {
    case F32: return p_embed_elem<F32>(a, token, col);
    case F16: return p_embed_elem<F16>(a, token, col);
    case Q4_0: return p_embed_elem<Q4_0>(a, token, col);
    case Q8_0: return p_embed_elem<Q8_0>(a, token, col);
    case Q4_K: return p_embed_elem<Q4_K>(a, token, col);
    case Q5_K: return p_embed_elem<Q5_K>(a, token, col);
    default: return p_embed_elem<Q6_K>(a, token, col);
  }
}

// ------------------------------------------------------------------ kernel

struct Ring {
  uint64_t *full, *empty;  // weight slots: bytes landed / the stage's results read (epilogue warp)
  uint64_t *done;          // chunk results (P_RES_STAGES): written by every compute warp
  uint8_t *slots;
  int ns;
};

// Waits for phase `par` of mbarrier b. False when the grid is winding down or this
// wait ran out (then status[0] = 1 and the stop flag is raised).
__device__ __noinline__ bool mbar_wait_slow(uint64_t *b, unsigned par, volatile int *stop, int *status) {
  const uint64_t t0 = gtime();
#ifdef WGD_PERSIST_TRACE
  struct Acc {
    uint64_t t0;
    __device__ ~Acc() {
      if (threadIdx.x == 0 && (blockIdx.x == 0 || blockIdx.x == 100)) g_wait_acc[blockIdx.x == 0 ? 0 : 1] += gtime() - t0;
    }
  } acc_guard{t0};
#endif
  while (!mbar_try(b, par)) {
    if (*stop) return false;
    if (gtime() - t0 > P_TIMEOUT_NS) {
      atomicCAS(status, 0, 1);
      *stop = 1;
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ bool mbar_wait(uint64_t *b, unsigned par, volatile int *stop, int *status) {
  return mbar_test(b, par) || mbar_wait_slow(b, par, stop, status);
}

// Barrier over every CTA of every rank of a tensor-parallel group, after this CTA's partial rows
// were pushed to the peers. Two levels: every CTA makes its peer stores visible (system-scope
// fence) and arrives on its rank's local counter (bar[1]); CTA 0 waits for the rank's CTAs, adds 1
// to the arrival counter in every rank's exchange buffer (one system-scope release per rank instead
// of one per CTA), waits until its own rank's counter holds every rank's arrival, and releases the
// rank's CTAs through a local generation word (bar[2]). The counters only grow (the exchange
// counter across launches too: xbase is its count before this launch), so no reset races a faster
// peer. A wait that runs out (x_limit_ns) raises the status; CTA 0 releases its rank's CTAs also then.
__device__ bool x_sync(const PersistArgs &a, unsigned &xgen, volatile int *stop) {
  bar_all();
  if (threadIdx.x == 0 && !*stop) {
    __threadfence_system();
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.bar + 1) : "memory");
    const uint64_t t0 = gtime();
    if (blockIdx.x == 0) {
      bool ok = true;
      const unsigned lt = (xgen + 1u) * gridDim.x;
      for (unsigned it = 1; (int)(ld_acquire(a.bar + 1) - lt) < 0; it++)
        if ((it & 63) == 0 && (*(volatile int *)a.status == 1 || gtime() - t0 > a.x_limit_ns)) {
          ok = false;
          break;
        }
      if (ok) {
        __threadfence_system();
        for (int j = 0; j < a.tp; j++)
          asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(a.xbuf[j] + a.x_bar) : "memory");
        const unsigned target = a.xbase + (xgen + 1u) * (unsigned)a.tp;
        const unsigned *ctr = reinterpret_cast<const unsigned *>(a.xbuf[a.rank] + a.x_bar);
        for (unsigned it = 1;; it++) {
          unsigned v;
          asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
          if ((int)(v - target) >= 0) break;
          if ((it & 63) == 0 && (*(volatile int *)a.status == 1 || gtime() - t0 > a.x_limit_ns)) {
            ok = false;
            break;
          }
        }
      }
      if (!ok) {
        atomicCAS(a.status, 0, 1);
        *stop = 1;
      }
      asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(a.bar + 2), "r"(xgen + 1u) : "memory");
    } else {
      for (unsigned it = 1; (int)(ld_acquire(a.bar + 2) - (xgen + 1u)) < 0; it++)
        if ((it & 63) == 0 && gtime() - t0 > a.x_limit_ns + P_TIMEOUT_NS) {
          atomicCAS(a.status, 0, 1);
          break;
        }
      if (*(volatile int *)a.status == 1) *stop = 1;
    }
    xgen++;
  }
  if (threadIdx.x == 0) stop[3] = *stop;
  bar_all();
  return !stop[3];
}

// Grid barrier for the compute and epilogue warps of every CTA. Returns false when
// the grid is winding down. Every such warp reaches every call, also after a failed
// wait, so no named barrier is left waiting.
__device__ bool grid_sync(const PersistArgs &a, unsigned &gen, volatile int *stop) {
  bar_all();
#ifdef WGD_PERSIST_TRACE
  int tr_i = -1;
  if (threadIdx.x == 0 && blockIdx.x < 160) {
    tr_i = g_bar_index[blockIdx.x]++;
    if (tr_i >= 0 && tr_i < TR_BARS) g_bars[blockIdx.x][tr_i][0] = gtime();
  }
#endif
  if (threadIdx.x == 0 && !*stop) {
    // The CTA's writes are ordered before thread 0's release by the barrier above. The
    // arrival counter only grows within a launch (zeroed before it): barrier number gen
    // is complete when it reaches (gen + 1) * grid, which every CTA reads directly.
    const unsigned target = (gen + 1u) * gridDim.x;
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.bar) : "memory");
    const uint64_t t0 = gtime();
    for (unsigned it = 1; (int)(ld_acquire(a.bar) - target) < 0; it++) {
      if ((it & 63) == 0 && (*(volatile int *)a.status == 1 || gtime() - t0 > P_TIMEOUT_NS)) {
        atomicCAS(a.status, 0, 1);
        *stop = 1;
        break;
      }
    }
    gen++;
  }
#ifdef WGD_PERSIST_TRACE
  if (threadIdx.x == 0 && tr_i >= 0 && tr_i < TR_BARS) g_bars[blockIdx.x][tr_i][1] = gtime();
#endif
  // one snapshot of the stop flag (the producer may raise it at any time) so that
  // every thread takes the same branch after this barrier
  if (threadIdx.x == 0) stop[3] = *stop;
  bar_all();
  return !stop[3];
}

// Cursor over the ring stages of this CTA, in execution order: (step, GEMV phase, first unit).
struct SIt {
  int step, p, u0, s0, u1, k, CB;
  const uint8_t *w;
};
__device__ bool sit_seek(const PersistArgs &a, int grid, int c, SIt &it) {
  for (; it.step < a.steps; it.step++, it.p = 0) {
    for (; it.p < a.nphases; it.p++) {
      const PPhase &ph = a.phases[it.p];
      if (ph.kind != PH_GEMV) continue;
      int u0, u1;
      unit_range(ph.g.tiles, ph.g.nkb, grid, c, u0, u1);
      if (u0 >= u1) continue;
      it.u0 = it.s0 = u0;
      it.u1 = u1;
      it.k = slot_units(ph.g.type);
      it.CB = chunk_bytes(ph.g.type);
      it.w = ph.g.w;
      return true;
    }
  }
  return false;
}
__device__ bool sit_next(const PersistArgs &a, int grid, int c, SIt &it) {
  it.s0 += it.k;
  if (it.s0 < it.u1) return true;
  it.p++;
  return sit_seek(a, grid, c, it);
}


__device__ __forceinline__ void prefetch_l2(const void *src, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Producer (lane 0 of warp 15): every weight chunk of this CTA, in execution order,
// into the ring; optionally the same stream a.l2_ahead stages earlier into L2, so
// HBM keeps streaming while the other warps wait at barriers.
__device__ void producer(const PersistArgs &a, const Ring &R, volatile int *stop) {
  if ((threadIdx.x & 31) != 0) return;
  const int grid = gridDim.x, c = blockIdx.x;
  SIt f{0, 0, 0, 0, 0, 0, 0, nullptr};
  SIt pf = f;
  bool fv = sit_seek(a, grid, c, f), pv = sit_seek(a, grid, c, pf);
  int ahead = 0;
  unsigned g = 0, epar = 1u;  // stages issued; the parity that frees the current slot
  int slot = 0;
  while (fv) {
    while (pv && ahead < a.l2_ahead) {
      prefetch_l2(pf.w + (size_t)pf.s0 * pf.CB, (unsigned)(min(pf.k, pf.u1 - pf.s0) * pf.CB));
      pv = sit_next(a, grid, c, pf);
      ahead++;
    }
#ifdef WGD_PERSIST_TRACE
    const uint64_t tw0 = gtime();
#endif
    if (!mbar_wait(R.empty + slot, epar, stop, a.status)) break;
#ifdef WGD_PERSIST_TRACE
    // time this producer waited for a free slot, per phase (slot 7)
    if ((blockIdx.x == 0 || blockIdx.x == 100) && f.step < TR_STEPS && f.p < TR_PHASES) {
      uint64_t &w = g_trace[blockIdx.x == 0 ? 0 : 1][f.step][f.p][7];
      w = (f.s0 == f.u0 ? 0 : w) + (gtime() - tw0);
    }
#endif
    const int n = min(f.k, f.u1 - f.s0);
    if (f.s0 == f.u0) P_TRACE(f.step, f.p, 4);
    if (f.s0 + f.k >= f.u1) P_TRACE(f.step, f.p, 5);
    mbar_expect_tx(R.full + slot, (unsigned)(n * f.CB));
    bulk_g2s(R.slots + (size_t)slot * P_SLOT_BYTES, f.w + (size_t)f.s0 * f.CB, (unsigned)(n * f.CB), R.full + slot);
    g++;
    if (++slot == R.ns) {
      slot = 0;
      epar ^= 1u;
    }
    fv = sit_next(a, grid, c, f);
    ahead--;
  }
  // copies issued but not consumed (an early stop) must land before the CTA exits
  const unsigned first = g > (unsigned)R.ns ? g - R.ns : 0u;
  for (unsigned q = first; q < g; q++) {
    const uint64_t t0 = gtime();
    while (!mbar_test(R.full + q % R.ns, (q / R.ns) & 1u)) {
      if (gtime() - t0 > P_TIMEOUT_NS) break;
      __nanosleep(64);
    }
  }
}

// One warp copies a phase descriptor from the plan in global memory into shared memory.
__device__ __forceinline__ void p_copy_phase(PPhase *dst, const PPhase *src, int lane) {
  static_assert(sizeof(PPhase) % 4 == 0, "descriptor copied in words");
  const uint32_t *s = reinterpret_cast<const uint32_t *>(src);
  uint32_t *d = reinterpret_cast<uint32_t *>(dst);
  for (int i = lane; i < (int)(sizeof(PPhase) / 4); i += 32) d[i] = __ldg(s + i);
}

__global__ void __launch_bounds__(P_THREADS, 1) persist_kernel(const PersistArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  Ring R;
  R.ns = a.nstage;
  R.full = reinterpret_cast<uint64_t *>(smem);
  R.empty = R.full + P_MAXSTAGES;
  R.done = R.empty + P_MAXSTAGES;
  R.slots = smem + 256;
  uint8_t *xs = R.slots + (size_t)R.ns * P_SLOT_BYTES;
  PShared &sh = *reinterpret_cast<PShared *>(xs + a.xs_bytes);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    for (int i = 0; i < R.ns; i++) {
      mbar_init(R.full + i, 1);
      mbar_init(R.empty + i, 1);
    }
    for (int i = 0; i < P_RES_STAGES; i++) {
      mbar_init(R.done + i, P_CWARPS);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (tid < 4) sh.flags[tid] = 0;
  __syncthreads();
  volatile int *stop = &sh.flags[0];
  if (warp == P_PWARP) {
    producer(a, R, stop);
    return;
  }

  // ---------------- compute warps (0..13) and the epilogue warp (14)
  const bool comp = warp < P_CWARPS, epi = warp == P_EWARP;
  const int grid = gridDim.x, c = blockIdx.x;
  unsigned gen = 0;   // grid barriers passed in this launch (thread 0)
  unsigned xgen = 0;  // cross-rank barriers passed in this launch (thread 0; tensor parallelism)
  unsigned g = 0;  // ring stage counter, in step with the producer
  // the first two phase descriptors; later ones are copied one phase ahead of use
  if (epi) {
    p_copy_phase(&sh.dsc[0], a.phases, lane);
    p_copy_phase(&sh.dsc[1], a.phases + (a.nphases > 1 ? 1 : 0), lane);
  }
  int token = a.dev_first ? __ldcg(a.dev_first) : a.first;
  const int start = a.dev_start ? __ldcg(a.dev_start) : a.start;
  bool att_staged = false;  // attention stage 0 was filled during the previous phase
  for (int step = 0; step < a.steps; step++) {
    const int pos = start + step;
    // embedding row of the token (engine.ts:140-145), spread over the CTAs
    if (comp) {
      const int per = (a.hidden + grid - 1) / grid;
      const int lo = c * per, hi = min(a.hidden, lo + per);
      for (int e = lo + tid; e < hi; e += P_CWARPS * 32) a.x[e] = p_embed_value(a, token, e) * a.embd_scale;
    }
    if (!grid_sync(a, gen, stop)) break;
    bool alive = true;
    for (int p = 0; p < a.nphases && alive; p++) {
      const int q = step * a.nphases + p;  // position in the phase sequence of the launch
      const PPhase &ph = sh.dsc[q % 3];
      if (epi) p_copy_phase(&sh.dsc[(q + 2) % 3], a.phases + (p + 2) % a.nphases, lane);
      if (tid == 0) P_TRACE(step, p, 0);
      if (ph.kind == PH_ATTN) {
        const PAttn &A = ph.a;
        int chunk, nsp;
        attn_split(A, pos, a.nsp_max, chunk, nsp);
        const int items = A.kv_heads * nsp;
        if (comp)
          for (int it = c; it < items; it += grid)
            if (A.hd % 32 == 0)
              p_attn_item<8>(A, pos, it / nsp, it % nsp, nsp, chunk, a.nsp_max, reinterpret_cast<float *>(xs), a.att_part,
                             a.att_ctr, &sh.flags[1], it == c && att_staged, step, p);
            else
              p_attn_item<4>(A, pos, it / nsp, it % nsp, nsp, chunk, a.nsp_max, reinterpret_cast<float *>(xs), a.att_part,
                             a.att_ctr, &sh.flags[1], it == c && att_staged, step, p);
        att_staged = false;
        if (tid == 0) P_TRACE(step, p, 3);
        alive = grid_sync(a, gen, stop);
        continue;
      }
      // ---- GEMV phase
      const PGemv &pg = ph.g;
      const int nkb = pg.nkb, k = slot_units(pg.type), CB = chunk_bytes(pg.type);
      int u0, u1;
      unit_range(pg.tiles, nkb, grid, c, u0, u1);
      if (comp) {
        const bool q6 = pg.type == Q6_K;
        const PX X = px_carve(xs, pg.cols);
        if (pg.xsum) {
          // the summed row (residual plus the ranks' partials) sits behind the digit records in xs
          const float *part = reinterpret_cast<const float *>(a.xbuf[a.rank] + a.x_slot) +
                              (size_t)(pg.xsum - 1) * P_TP_MAX * a.hidden;
          float *row = reinterpret_cast<float *>(xs + ((px_bytes(pg.cols) + 15) & ~(size_t)15));
          p_sum_parts(pg.x, part, a.tp, a.hidden, pg.cols, row, pg.x_out);
          p_digitise<true>(row, pg.norm_w, pg.eps, pg.cols, q6, X, sh.red, sh.dsum[warp], warp, lane);
        } else {
          p_digitise<false>(pg.x, pg.norm_w, pg.eps, pg.cols, q6, X, sh.red, sh.dsum[warp], warp, lane);
        }
        bar_comp();
        if (tid == 0) P_TRACE(step, p, 1);
        // when attention follows, warps 0..3 start copying this CTA's first K/V tile now (rows
        // of earlier positions only) into attention stage 0, above the digit records; issued after
        // the digitisation so that its loads of the phase input do not queue behind these copies
        if (p + 1 < a.nphases && sh.dsc[(q + 1) % 3].kind == PH_ATTN && warp < 4) {
          const PAttn &A = sh.dsc[(q + 1) % 3].a;
          // (only where the digit records end below stage 0; a tensor-parallel input row behind them
          // is no longer read once the records are written)
          if (px_bytes(pg.cols) <= (size_t)attn_stage_floats(A.hd) * 4) {
            int chunk, nsp;
            attn_split(A, pos, a.nsp_max, chunk, nsp);
            if (c < A.kv_heads * nsp) {
              const int kh = c / nsp, sp = c % nsp;
              const int end = pos + 1, begin = end - (end < A.window ? end : A.window);
              const int p0 = begin + sp * chunk, p1 = min(end, p0 + chunk);
              p_attn_stage(A, pos, kh, p1, p0, reinterpret_cast<float *>(xs), 0, tid, 4);
              att_staged = true;
            }
          }
        }
        const PLane PL = p_lane(lane);
        // this warp's chunks: u0 + warp, u0 + warp + P_CWARPS, ... (tile t, super-block kb)
        int nu = u0 + warp, kb = nkb ? nu % nkb : 0;
        // ring slot and its fill parity, advanced with g (no division per stage)
        int slot = (int)(g % (unsigned)R.ns);
        unsigned fpar = (g / (unsigned)R.ns) & 1u;
        for (int s0 = u0; s0 < u1; s0 += k, g++) {
          const int s1 = min(u1, s0 + k), rs = g % P_RES_STAGES;
          // this warp's chunk of the stage (at most one: k <= P_CWARPS). After the reduction over the
          // four lanes of an MMA row group, lane 4i holds row i and lane 4i+1 row i+8.
          float v = 0.f;
          const bool mine = nu < s1;
          const int at = nu - s0;
          const bool ok = mbar_wait(R.full + slot, fpar, stop, a.status);
          if (ok) {
            if (mine) {
              float acc[2] = {0.f, 0.f};
              const uint8_t *cp = R.slots + (size_t)slot * P_SLOT_BYTES + (size_t)at * CB;
              if (q6) p_q6k(cp, kb, X, PL, lane, acc);
              else p_q4k(cp, kb, X, PL, lane, acc);
              // (a0 + a1) + (a2 + a3) for each row, as two shuffles: even lanes keep row i, odd
              // lanes row i+8, and each sends the other row's partial to its neighbour
              const bool odd = lane & 1;
              v = odd ? acc[1] : acc[0];
              v += __shfl_xor_sync(0xffffffffu, odd ? acc[0] : acc[1], 1);
              v += __shfl_xor_sync(0xffffffffu, v, 2);
              kb += P_CWARPS;
              while (kb >= nkb) kb -= nkb;
            }
          }
          if (mine) nu += P_CWARPS;
          // (result stage rs is free: this stage's weights were issued after the epilogue warp read
          // stage g - ns, and ns <= P_RES_STAGES)
          if (ok && mine && (lane & 3) < 2) sh.res[rs][at][(lane >> 2) + 8 * (lane & 1)] = v;
          __syncwarp();
          if (lane == 0) mbar_arrive(R.done + rs);
          if (++slot == R.ns) {
            slot = 0;
            fpar ^= 1u;
          }
        }
        if (tid == 0) P_TRACE(step, p, 2);
#ifdef WGD_PERSIST_TRACE
        if (tid == 0 && (blockIdx.x == 0 || blockIdx.x == 100) && step < TR_STEPS) {
          g_trace[blockIdx.x == 0 ? 0 : 1][step][p][6] = g_wait_acc[blockIdx.x == 0 ? 0 : 1];
          g_wait_acc[blockIdx.x == 0 ? 0 : 1] = 0;
        }
#endif
      } else {
        // epilogue warp: tile sums in k-block order, then the tile's epilogue
        GemvCtx C;
        C.g = &pg;
        C.a = &a;
        C.best_v = -FLT_MAX;
        C.best_i = -1;
        C.row0 = a.tp > 1 && pg.argmax ? a.vocab0 : 0;
        int t = nkb ? u0 / nkb : 0, kbe = 0;
        // the residual rows this CTA will add into are final before the phase starts (only this CTA
        // writes them in it): load them now, off the phase's tail
        C.pre_t0 = t;
#pragma unroll
        for (int k2 = 0; k2 < P_PRE; k2++) {
          const int row = (t + k2) * 16 + lane;
          C.pre[k2] = pg.epi == EPI_ADD && lane < 16 && (t + k2) * nkb < u1 && row < pg.rows ? __ldcg(pg.y + row) : 0.f;
        }
        float run = 0.f;
        int eslot = (int)(g % (unsigned)R.ns);  // the weight slot of stage g
        for (int s0 = u0; s0 < u1; s0 += k, g++) {
          const int n = min(k, u1 - s0), rs = g % P_RES_STAGES, ws = eslot;
          if (++eslot == R.ns) eslot = 0;
          if (mbar_wait(R.done + rs, (g / P_RES_STAGES) & 1u, stop, a.status)) {
            float v[P_STAGE_UNITS];
#pragma unroll
            for (int j = 0; j < P_STAGE_UNITS; j++) v[j] = (j < n && lane < 16) ? sh.res[rs][j][lane] : 0.f;
            __syncwarp();
            // every compute warp is done with the weight slot and the results are read: the
            // producer may refill the slot (and the result stage is free once it has)
            if (lane == 0) mbar_arrive(R.empty + ws);
            if (nkb >= 8) {
              // the stage's results in k-block order; a tile ends where the running k-block count
              // reaches nkb. With n <= 16 results and nkb >= 8 a stage holds at most two tile ends,
              // so the sums run branch-free and the epilogue is emitted after the loop (the same
              // additions in the same order as one epilogue per result)
              const int e1 = nkb - 1 - kbe, e2 = e1 + nkb;
              float o1 = 0.f, o2 = 0.f;
#pragma unroll
              for (int j = 0; j < P_STAGE_UNITS; j++) {
                if (j < n) {
                  run += v[j];
                  if (j == e1) { o1 = run; run = 0.f; }
                  if (j == e2) { o2 = run; run = 0.f; }
                }
              }
              if (e1 < n) p_epilogue(C, t++, o1, lane);
              if (e2 < n) p_epilogue(C, t++, o2, lane);
              kbe += n;
              while (kbe >= nkb) kbe -= nkb;
            } else {
              // narrow inputs (tensor-parallel shards): several tile ends per stage
#pragma unroll
              for (int j = 0; j < P_STAGE_UNITS; j++) {
                if (j < n) {
                  run += v[j];
                  if (++kbe == nkb) {
                    p_epilogue(C, t++, run, lane);
                    run = 0.f;
                    kbe = 0;
                  }
                }
              }
            }
          } else {
            __syncwarp();
            if (lane == 0) mbar_arrive(R.empty + ws);
          }
        }
        if (lane == 0) P_TRACE(step, p, 3);
        if (pg.argmax) {
          float bv = C.best_v;
          int bi = C.best_i;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
          }
          if (lane == 0) {
            const bool stop_req = c == 0 && a.cancel && *(volatile const int *)a.cancel;
            if (a.tp > 1) {
              // every rank's candidate table (two by token parity); rank 0's cancel word rides along
              // so that every rank stops after the same token
              const unsigned par = (a.xstep0 + (unsigned)step) & 1u;
              for (int j = 0; j < a.tp; j++) {
                float2 *pc = reinterpret_cast<float2 *>(a.xbuf[j] + a.x_cand) + ((size_t)par * P_TP_MAX + a.rank) * P_CAND_STRIDE;
                pc[c] = make_float2(bv, __int_as_float(bi));
                if (c == 0 && a.rank == 0) pc[grid] = make_float2(stop_req ? 1.f : 0.f, 0.f);
              }
            } else {
              __stcg(a.cand + c, make_float2(bv, __int_as_float(bi)));
              if (stop_req) atomicExch(a.status + 2, 1);
            }
          }
        }
      }
      // after a pushed partial (O, down) or the LM head's candidates, every rank of the group meets
      alive = a.tp > 1 && (pg.push || pg.argmax) ? x_sync(a, xgen, stop) : grid_sync(a, gen, stop);
    }
    if (!alive) break;
    // greedy token: the best candidate of all CTAs (every CTA computes the same)
    {
      float bv = -FLT_MAX;
      int bi = -1;
      const float2 *cand = a.cand;
      int ncand = grid;
      if (a.tp > 1) {  // every rank's CTAs, in this rank's buffer
        cand = reinterpret_cast<const float2 *>(a.xbuf[a.rank] + a.x_cand) +
               (size_t)((a.xstep0 + (unsigned)step) & 1u) * P_TP_MAX * P_CAND_STRIDE;
        ncand = a.tp * P_CAND_STRIDE;
      }
      for (int i = tid; i < ncand; i += (P_CWARPS + 1) * 32) {
        if (a.tp > 1 && i % P_CAND_STRIDE >= grid) continue;  // control words and unused slots
        const float2 cv = __ldcg(cand + i);
        const int ci = __float_as_int(cv.y);
        if (better(cv.x, ci, bv, bi)) { bv = cv.x; bi = ci; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
      }
      if (lane == 0) sh.best[warp] = make_float2(bv, __int_as_float(bi));
      bar_all();
      if (tid == 0) {
        float v = -FLT_MAX;
        int i = -1;
        for (int w = 0; w <= P_CWARPS; w++) {
          const float ov = sh.best[w].x;
          const int oi = __float_as_int(sh.best[w].y);
          if (better(ov, oi, v, i)) { v = ov; i = oi; }
        }
        sh.flags[2] = i;
      }
      bar_all();
      token = sh.flags[2];
      const bool cancelled = a.tp > 1 ? __ldcg(cand + grid).x != 0.f : __ldcg(a.status + 2) != 0;
      if (c == 0 && tid == 0) {
        a.tokens[step] = token;
        a.status[1] = step + 1;
        if (token < 0) atomicCAS(a.status, 0, 2);
        else if (cancelled && step + 1 < a.steps) atomicCAS(a.status, 0, 3);
      }
      if (token < 0 || cancelled) break;
    }
  }
  if (tid == 0) *stop = 1;  // releases a producer still waiting for a free slot
  (void)epi;
}

}  // namespace

#ifdef WGD_PERSIST_TRACE
extern "C" __attribute__((visibility("default"))) int wgd_debug_persist_trace(uint64_t *out, size_t n) {
  const size_t bytes = sizeof(g_trace) < n * sizeof(uint64_t) ? sizeof(g_trace) : n * sizeof(uint64_t);
  return (int)cudaMemcpyFromSymbol(out, g_trace, bytes);
}
extern "C" __attribute__((visibility("default"))) int wgd_debug_persist_bars(uint64_t *out, int reset) {
  if (reset) {
    static int zeros[160] = {0};
    return (int)cudaMemcpyToSymbol(g_bar_index, zeros, sizeof(zeros));
  }
  return (int)cudaMemcpyFromSymbol(out, g_bars, sizeof(g_bars));
}
#endif

// ------------------------------------------------------------------ host side

static int attn_smem_bytes(int group, int hd) {
  // K|V stages, q, new k and v rows, score parts [AW][8][32], probabilities [32][8], head state [3][8]
  return 4 * (group * hd + 2 * hd + 2 * 2 * 32 * (hd + 4) + AW_MAX * 8 * 32 + 32 * 8 + 3 * 8);
}

size_t persist_smem_bytes(int max_cols, int group, int hd, int nstage, int *xs, int row_cols) {
  size_t x = px_bytes(max_cols);
  const size_t at = (size_t)attn_smem_bytes(group, hd);
  if (at > x) x = at;
  if (row_cols > 0) {
    const size_t r = ((px_bytes(row_cols) + 15) & ~(size_t)15) + 4 * (size_t)row_cols;
    if (r > x) x = r;
  }
  x = (x + 127) & ~(size_t)127;
  if (xs) *xs = (int)x;
  return 256 + (size_t)nstage * P_SLOT_BYTES + x + sizeof(PShared);
}

int persist_max_stages(int max_cols, int group, int hd, int row_cols) {
  const size_t limit = 227 * 1024;
  const size_t fixed = persist_smem_bytes(max_cols, group, hd, 0, nullptr, row_cols);
  if (fixed >= limit) return 0;
  int ns = (int)((limit - fixed) / P_SLOT_BYTES);
  return ns > P_MAXSTAGES ? P_MAXSTAGES : ns;
}

cudaError_t launch_persist(const PersistArgs &a, int grid, cudaStream_t s) {
  const size_t smem = 256 + (size_t)a.nstage * P_SLOT_BYTES + (size_t)a.xs_bytes + sizeof(PShared);
  static size_t attr = 0;
  if (attr < smem) {
    cudaError_t e = cudaFuncSetAttribute(persist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(P_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr1[1];
  attr1[0].id = cudaLaunchAttributeCooperative;
  attr1[0].val.cooperative = 1;
  cfg.attrs = attr1;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, persist_kernel, a);
}

}  // namespace wgd
