// decode_step.cuh -- phase table of the persistent decode-step kernel.
#pragma once
#include <cuda_fp16.h>

#include "kernels.cuh"

namespace ch {

enum PhaseKind : uint32_t { PH_GEMV = 0, PH_ATTN = 1, PH_TOPK = 2, PH_MERGE = 3 };
// how a GEMV phase builds its input vector
enum PrologueMode : uint32_t {
  PM_DIRECT = 0,    // x_in as is (attention output)
  PM_NORM = 1,      // rmsnorm(x_in) * norm_w                      (layer-0 input norm)
  PM_ADD_NORM = 2,  // x = (x_in + [rmsnorm(r) * post_w]) * scalar; rmsnorm(x) * norm_w
  PM_GELU = 3,      // gelu_tanh(gate) * up from an interleaved gate|up GEMV output
};

constexpr uint32_t kMaxWorld = 8;  // ranks of a tensor-parallel decode

// How a GEMV phase's tiles (row tiles x KT k tiles, row-tile major) are split over
// the grid's warps.  Stream-K: one balanced split over all grid*warps warps (row
// tiles may straddle CTAs).  Aligned: whole row tiles per CTA (rq or rq+1), then a
// balanced split over the CTA's warps -- no row tile crosses a CTA, so every
// output row is finished inside one CTA (used when outputs go to other GPUs).
struct Partition {
  uint32_t KT;        // k tiles per row tile
  uint32_t q, rem;    // stream-K: tiles per warp (q or q+1)
  uint32_t aligned;   // 1: whole row tiles per CTA
  uint32_t rq, rrem;  // aligned: row tiles per CTA (rq or rq+1)
};

// Output of a GEMV phase.  A row tile whose k tiles all fall in one CTA's share
// is finished by that CTA in `direct`; a row tile that straddles CTAs is left as
// one partial sum per CTA (slot 0: the CTA's first row tile, slot 1: its last)
// and the consumer phase adds them up while it loads its input.
struct GemvOut {
  float *direct;   // [rows]; act mode: B fragments (f16 hi|lo) of the rows/2 values gelu(gate) * up
  float *partial;  // [grid][2][16] CTA partial sums of straddling row tiles
  Partition pt;    // the producing GEMV's split
  uint32_t act;    // 1: interleaved gate|up GEMV whose consumer takes B fragments of gelu(gate) * up
  uint32_t row0;   // push 1: index of this rank's first row (act value) in the gathered vector;
                   // push 2: length of the exchanged vector
  uint32_t push;   // 1: rows go to every rank's copy of `direct` (peer stores), 0: local only,
                   // 2: low-latency exchange -- `direct` is a [2 parities][world][row0] array of
                   // 8-byte {value, epoch} words, one plain store per row and rank, no fence
  uint32_t xidx;   // push 2: index of this exchange within the launch (epoch = base[2] + xidx + 1)
  uint32_t kind;   // which of the launch's kKinds partitions (MegaArgs::kpart) produced it
};
constexpr uint32_t kKinds = 5;  // GEMV partitions of a launch: q|k|v, o, gate|up, down, LM head

struct alignas(16) Phase {
  uint32_t kind, fmt, pm, is_sliding;
  // barrier after this phase: cross = 1 when other ranks read its outputs (tensor
  // parallel); gidx = number of cross-rank barriers up to and including this one
  uint32_t cross, gidx;
  // nobar = 1: no barrier after this phase (its outputs are exchange words that the
  // consumers poll); lidx = grid barriers up to and including this one
  uint32_t nobar, lidx;
  // PM_ADD_NORM input: nsum > 1 = r_in.direct holds nsum partial vectors of K floats
  // (one per rank, row-parallel GEMV), added in rank order by the prologue
  uint32_t nsum;
  // GEMV
  const uint8_t *tiles;
  uint32_t row_tiles, k_tiles, K, vocab, vocab0;
  GemvOut out;
  // GEMV prologue inputs / ATTN and TOPK inputs
  const float *x_in;
  GemvOut r_in;
  const float *post_w, *norm_w;
  float scalar, attn_scale;
  float *x_out, *normed_out;
  // ATTN
  const float *q_norm_w, *k_norm_w;
  const float2 *rope_cs;
  __half *k_cache, *v_cache;
  float *attn_out;  // ATTN output, written as B fragments (f16 hi|lo) of the o-projection's input
};

// the weight stream of one GEMV phase (phases in order, GEMV phases only)
struct alignas(16) StreamDesc {
  const uint8_t *tiles;
  Partition pt;
};

struct MegaArgs {
  const Phase *phases;
  const StreamDesc *streams;
  uint32_t nstreams;
  Partition kpart[kKinds];  // the partition of each GEMV kind (GemvOut::kind)
  uint32_t nphases, grid;
  unsigned long long *arrive;  // this GPU's grid-barrier arrivals (monotonic across launches)
  unsigned long long *base;    // [3] arrivals (local, cross-rank) and exchange epochs before this
                               // launch (advanced by the launch)
  unsigned long long *garrive; // tensor parallel: rank arrivals of cross-rank barriers (in the arena)
  uint32_t ncross;             // cross-rank barriers per launch
  uint32_t nlocal;             // grid barriers per launch (transitions with nobar = 0)
  uint32_t nx;                 // low-latency exchanges per launch
  uint32_t *err;
  const StepParams *sp;
  StepParams *sp_rw;  // device loop: the top-k phase records the token at history slot sp->step (else null)
  uint32_t nq, nkv, rot, attn_max_splits, cache_slots;  // nq / nkv: this rank's heads
  float eps;
  float *attn_partial;
  uint32_t *attn_counters;
  uint64_t *topk_cand;
  uint32_t *topk_counter;
  uint32_t *ids;
  float *vals;
  uint32_t *token_out, *token_hist;
  uint32_t hist_cap;
  // tensor parallel (world > 1): every rank's exchange arena, mapped into this process
  uint32_t world, rank;
  uint32_t attn_q0;            // global index of this rank's first q head
  uint32_t attn_local;         // tensor parallel: the attention output stays on this rank (row-parallel o)
  uint8_t *arena[kMaxWorld];   // arena[rank] is this rank's own
  uint64_t *xcand;             // this rank's [world][64] top-64 candidates of every rank (in its arena)
};

int mk_warps();
constexpr uint32_t kMkMaxSplits = 24;  // attention splits per kv head held in registers by the combine
size_t mk_smem_bytes(uint32_t max_k, uint32_t hidden, uint32_t ratio, uint32_t max_splits, uint32_t cache_slots,
                     uint32_t grid);
cudaError_t launch_decode_step(const MegaArgs &a, size_t smem, cudaStream_t s);

}  // namespace ch
