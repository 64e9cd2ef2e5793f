// decode_step.cuh -- phase table of the persistent decode-step kernel.
#pragma once
#include <cuda_fp16.h>

#include "kernels.cuh"

namespace ch {

enum PhaseKind : uint32_t { PH_GEMV = 0, PH_ATTN = 1, PH_TOPK = 2 };
// how a GEMV phase builds its input vector
enum PrologueMode : uint32_t {
  PM_DIRECT = 0,    // x_in as is (attention output)
  PM_NORM = 1,      // rmsnorm(x_in) * norm_w                      (layer-0 input norm)
  PM_ADD_NORM = 2,  // x = (x_in + [rmsnorm(r) * post_w]) * scalar; rmsnorm(x) * norm_w
  PM_GELU = 3,      // gelu_tanh(gate) * up from an interleaved gate|up GEMV output
};

// Output of a GEMV phase.  A row tile whose k tiles all fall in one CTA's share
// is finished by that CTA in `direct`; a row tile that straddles CTAs is left as
// one partial sum per CTA (slot 0: the CTA's first row tile, slot 1: its last)
// and the consumer phase adds them up while it loads its input.
struct GemvOut {
  float *direct;       // [rows]; act mode: B fragments (f16 hi|lo) of the rows/2 values gelu(gate) * up
  float *partial;      // [grid][2][16] CTA partial sums of straddling row tiles
  uint32_t KT;         // k tiles of the producing GEMV
  uint32_t q, rem;     // balanced partition of its rows/16*KT tiles over grid*warps
  uint32_t act;        // 1: interleaved gate|up GEMV whose consumer takes B fragments
};

struct alignas(16) Phase {
  uint32_t kind, fmt, pm, is_sliding;
  // GEMV
  const uint8_t *tiles;
  uint32_t row_tiles, k_tiles, K, q, rem, vocab;
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
  float *attn_out;  // ATTN output, written as B fragments of the o-projection's input
};

// the weight stream of one GEMV phase (phases in order, GEMV phases only)
struct alignas(16) StreamDesc {
  const uint8_t *tiles;
  uint32_t q, rem;  // balanced partition of the phase's tiles over grid * warps
};

struct MegaArgs {
  const Phase *phases;
  const StreamDesc *streams;
  uint32_t nstreams;
  uint32_t nphases, grid;
  unsigned long long *arrive;  // grid-barrier arrivals (monotonic across launches)
  uint32_t *epoch;    // completed launches
  uint32_t *err;
  const StepParams *sp;
  StepParams *sp_rw;  // device loop: step counter advanced by the top-k phase (else null)
  uint32_t nq, nkv, rot, attn_max_splits, cache_slots;
  float eps;
  float *attn_partial;
  uint32_t *attn_counters;
  uint64_t *topk_cand;
  uint32_t *topk_counter;
  uint32_t *ids;
  float *vals;
  uint32_t *token_out, *token_hist;
  uint32_t hist_cap;
};

int mk_warps();
constexpr uint32_t kMkMaxSplits = 24;  // attention splits per kv head held in registers by the combine
size_t mk_smem_bytes(uint32_t max_k, uint32_t hidden, uint32_t ratio, uint32_t max_splits, uint32_t cache_slots,
                     uint32_t grid);
cudaError_t launch_decode_step(const MegaArgs &a, size_t smem, cudaStream_t s);

}  // namespace ch
