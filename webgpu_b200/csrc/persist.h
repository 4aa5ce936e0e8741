// Persistent decode kernel: one cooperative launch runs whole decode tokens
// (embedding, every layer, LM head, greedy argmax, token feedback) with grid
// barriers between dependent phases instead of kernel boundaries.
//
// Each CTA (one per SM) has a producer warp that streams the CTA's share of
// every weight matrix, in execution order, through a ring of shared-memory
// slots with bulk async copies (cp.async.bulk + mbarrier transaction counts).
// The stream does not depend on activations, so it runs ahead across the
// barriers and keeps HBM busy while the consumer warps wait for the previous
// phase. Consumer warps digitise the phase input (RMSNorm fused) into
// shared memory and run the integer tensor-core GEMV of gemv2_impl.cuh on the
// staged chunks.
#pragma once
#include <cstdint>

#include <cuda_runtime.h>

namespace wgd {

enum PhaseKind { PH_GEMV = 0, PH_ATTN = 1 };
constexpr int P_TP_MAX = 8;  // ranks of a tensor-parallel group

struct PGemv {
  const uint8_t *w;  // tiled weights (Q4_K or Q6_K)
  int type, rows, cols, tiles, nkb;
  const float *x;       // input row (cols floats)
  const float *norm_w;  // RMSNorm weight applied to x first, or null
  float eps;
  float *y;
  const float *bias;
  int epi;     // Epi
  int argmax;  // track the greedy token over the outputs (LM head)
  // tensor parallelism: the input is x plus the tp partial rows of exchange slot xsum - 1
  // (xsum 0: x alone), summed in rank order; the sum is also stored to x_out (super-block sb by
  // CTA sb % grid) as the residual stream of the next phases. push > 0: the outputs are this
  // rank's partial rows, stored into slot push - 1 of every rank's exchange buffer.
  int xsum, push;
  float *x_out;
};

struct PAttn {
  const float *qkv;  // q heads | k heads | v heads of the decoded row
  float *k, *v;      // [kv_heads][capacity][hd] ring caches
  float *out;        // [heads][hd]
  const float *q_norm, *k_norm;
  const float2 *table;  // (cos, sin)[position][rot/2]
  int heads, kv_heads, hd, capacity, window, rot, mode;
  float scale, eps;
};

struct PPhase {
  int kind;
  PGemv g;
  PAttn a;
};

struct PersistArgs {
  const PPhase *phases;  // one token: layers' phases, then the LM head (argmax = 1)
  int nphases;
  // embedding row gather at the start of each token
  const uint8_t *embd;
  int embd_type, embd_tiled;
  int64_t embd_drow;
  int hidden, vocab;
  float embd_scale;
  float *x;  // hidden state [hidden]
  // tokens
  int first, start, steps;
  const int *dev_first, *dev_start;  // non-null: first token and position read from device memory
  int *tokens;          // [steps] greedy tokens
  const int *cancel;    // host-mapped flag polled between tokens, or null
  // scratch
  float *att_part;      // [kv_heads][nsp_max][group][hd + 4]
  unsigned *att_ctr;    // [kv_heads] (zero, left zero)
  float2 *cand;         // [grid] (best logit, index bits) of each CTA
  unsigned *bar;        // [0] grid-barrier arrivals, [1] cross-rank barrier arrivals of this rank's CTAs,
                        // [2] cross-rank barrier generations released to this rank's CTAs; zero at launch
  int *status;          // [0] 0 ok, 1 wait limit hit, 2 non-finite logits, 3 cancelled; [1] steps done
  int nstage, xs_bytes, nsp_max;
  int l2_ahead;  // ring stages requested into L2 ahead of the shared-memory copies (0: none)
  // tensor parallelism (tp > 1): every rank's exchange buffer (own included), mapped here
  int tp, rank, vocab0;
  char *xbuf[P_TP_MAX];
  unsigned long long x_bar, x_cand, x_slot;  // byte offsets of the kernel's region in an exchange buffer
  unsigned xbase;   // arrivals counted on this rank's cross-rank counter before this launch (one per rank and barrier)
  unsigned xstep0;  // tokens decoded by earlier launches of this group (candidate slot parity)
  unsigned long long x_limit_ns;  // bound of one cross-rank wait
};

constexpr int P_CWARPS = 14;                // compute warps (+ one epilogue warp, one producer warp)
constexpr int P_CAND_STRIDE = 256;          // candidate slots per rank in an exchange buffer (grid + 1 control word)
constexpr int P_THREADS = (P_CWARPS + 2) * 32;
constexpr int P_SLOT_BYTES = 32256;        // 14 Q4_K or 9 Q6_K tile chunks

// Shared-memory bytes for a plan whose GEMV inputs are at most max_cols wide and
// whose attention uses (group, hd); returns the xs region size in *xs.
// row_cols > 0 (tensor parallelism): room for a summed input row of that width behind the digit
// records of a row_cols-wide phase input.
size_t persist_smem_bytes(int max_cols, int group, int hd, int nstage, int *xs, int row_cols = 0);
int persist_max_stages(int max_cols, int group, int hd, int row_cols = 0);
// Cooperative launch on `grid` CTAs (one per SM).
cudaError_t launch_persist(const PersistArgs &a, int grid, cudaStream_t s);

}  // namespace wgd
