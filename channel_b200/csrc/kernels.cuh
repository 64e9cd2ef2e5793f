// kernels.cuh -- host-side launch interface of the device kernels (internal to
// libchannel_b200; the public boundary is include/channel_cuda.h).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace ch {

// ---------------------------------------------------------------------------
// repacked weight tiles: 16 rows x 64 k (Q4) or 16 rows x 32 k (Q8), 576 bytes:
// 512 bytes of mma A-fragments (lane-major, 16 B per lane) + 64 bytes of scales.
constexpr int kTileBytes = 576;
constexpr int kTileRows = 16;
constexpr int kQ4TileK = 64;
constexpr int kQ8TileK = 32;

enum WFmt { FMT_Q4 = 0, FMT_Q8 = 1 };
enum Epi { EPI_STORE = 0, EPI_GELU_MUL = 1 };
enum Pro { PRO_NONE = 0, PRO_RMSNORM = 1, PRO_ADD_RMSNORM = 2 };
enum RowMap { MAP_PLAIN = 0, MAP_GATEUP = 1 };

inline size_t q4_tile_bytes(uint32_t rows, uint32_t cols) {
  return (size_t)(rows / kTileRows) * (cols / kQ4TileK) * kTileBytes;
}
inline size_t q8_tile_bytes(uint32_t rows, uint32_t cols) {
  return (size_t)(rows / kTileRows) * (cols / kQ8TileK) * kTileBytes;
}

struct GemvArgs {
  const uint8_t *tiles = nullptr;
  uint32_t row_tiles = 0, k_tiles = 0, K = 0;
  const float *x = nullptr;       // input (PRO_NONE), or x / x_in for the norm prologues
  const float *r = nullptr;       // PRO_ADD_RMSNORM: branch output added to x_in
  const float *post_w = nullptr;  // PRO_ADD_RMSNORM: optional rmsnorm weight applied to r first
  const float *norm_w = nullptr;  // norm weight of the prologue
  float scalar = 1.0f, eps = 1e-6f;
  float *x_out = nullptr;       // PRO_ADD_RMSNORM: updated residual (written by CTA 0)
  float *normed_out = nullptr;  // optional copy of the normed input (written by CTA 0)
  float *y = nullptr;
  float *partial = nullptr;     // stream-K partials [grid*warps][2][16]
  uint32_t *counters = nullptr; // per row tile, zero between launches
  uint32_t *err = nullptr;
  uint32_t cta_rows = 0;         // set by launch_gemv: CTAs take whole row tiles (shared-memory combine)
};

struct GemvPlan {
  int fmt = FMT_Q4, epi = EPI_STORE, pro = PRO_NONE;
  int grid = 0;
};

// SM count of the CURRENT device (cached per device)
int num_sms();
// Opt `func` in to `smem` bytes of dynamic shared memory on the CURRENT device.
// cudaFuncSetAttribute is per device, so the granted size is remembered per
// (device, kernel) under a lock; a second GPU in the same process gets its own
// opt-in instead of inheriting the first one's.
cudaError_t ensure_smem_attr(const void *func, size_t smem);
// scratch sizes needed by gemv for a given grid
size_t gemv_partial_floats(int grid);
int gemv_default_grid();
cudaError_t launch_gemv(const GemvPlan &plan, const GemvArgs &a, cudaStream_t s, bool pdl);

// repack / generate
cudaError_t launch_repack_q4(const uint32_t *src_blocks, const uint32_t *src_blocks_b, uint32_t rows_out, uint32_t cols,
                             int rowmap, uint8_t *dst, cudaStream_t s);
cudaError_t launch_repack_q8(const uint32_t *src_blocks, uint32_t rows, uint32_t cols, uint8_t *dst, cudaStream_t s);
cudaError_t launch_gen_q4_blocks(uint32_t *dst, uint32_t rows, uint32_t cols, uint64_t tseed, float scale_std,
                                 cudaStream_t s);
// rows [row0, row0 + rows) of the same generated matrix (a tensor-parallel shard)
cudaError_t launch_gen_q4_rows(uint32_t *dst, uint32_t row0, uint32_t rows, uint32_t cols, uint64_t tseed,
                               float scale_std, cudaStream_t s);
// columns [col0, col0 + ncols) of all rows of the same seeded matrix (row-parallel shards)
cudaError_t launch_gen_q4_cols(uint32_t *dst, uint32_t rows, uint32_t cols, uint32_t col0, uint32_t ncols,
                               uint64_t tseed, float scale_std, cudaStream_t s);
cudaError_t launch_gen_bf16(uint16_t *dst, size_t n, uint64_t tseed, float mean, float std, cudaStream_t s);
cudaError_t launch_gen_f32(float *dst, size_t n, uint64_t tseed, float mean, float std, cudaStream_t s);
cudaError_t launch_bf16_to_f32(const uint16_t *src, float *dst, size_t n, cudaStream_t s);
cudaError_t launch_quantize_q8_rows(const uint16_t *src_bf16, uint32_t rows, uint32_t cols, uint32_t *dst,
                                    cudaStream_t s);
cudaError_t launch_quantize_q4_rows(const uint16_t *src_bf16, uint32_t rows, uint32_t cols, uint32_t *dst,
                                    cudaStream_t s);

// ---------------------------------------------------------------------------
// decode step state read by the kernels (updated by H2D copy or by step_begin)
struct StepParams {
  uint32_t clock, slot, n_active, n_sliding;
  const uint32_t *active;   // device list of physical slots (full-attention layers)
  const uint32_t *sliding;  // device list (sliding layers)
  uint32_t step;            // index of this step in the plan (token history slot)
  uint32_t next;            // device loop: plan index of the next step (advanced by step_begin)
  uint32_t force;           // plan entry: token + 1 to embed instead of the fed-back token (0: fed back)
  uint32_t pad;
};

struct AttnArgs {
  const float *qkv;      // q [nq*D] | k [nkv*D] | v [nkv*D] (raw projections)
  const float *q_norm_w, *k_norm_w;
  const float2 *rope_cs;  // [rot/2] (cos, sin) of clock * inv_freq for this layer's theta
  __half *k_cache, *v_cache;  // [4096][nkv*D]
  const StepParams *sp;
  int is_sliding;
  uint32_t nq, nkv, D, rot;
  float eps, scale;
  float *out;           // [nq*D]
  float *partial;       // [nkv][splits][ratio][D+2]
  uint32_t *counters;   // [nkv]
  uint32_t *err;
  uint32_t cache_slots; // 4096
  // Batched decode, one token per stream: token b = grid z uses sp[b], rope_cs + b *
  // rope_stride, qkv + b * qkv_stride, out + b * out_stride, the caches of stream
  // stream[b] (cache_stride elements apart) and its own partial / counter slices.
  // One token with zero strides is the single-stream case.
  uint32_t n_tok = 1;
  const uint32_t *stream = nullptr;  // [n_tok] (nullptr: every token uses the caches as given)
  size_t cache_stride = 0;
  uint32_t qkv_stride = 0, out_stride = 0, rope_stride = 0;
};
int attn_default_splits(uint32_t nkv);
size_t attn_partial_floats(uint32_t nkv, uint32_t ratio, uint32_t D, int splits);
cudaError_t launch_decode_attn(const AttnArgs &a, int splits, cudaStream_t s, bool pdl);

struct TopkArgs {
  const float *logits;
  uint32_t V;
  uint64_t *cand;      // [blocks][64] composite keys
  uint32_t *counter;   // 1 word, zero between launches
  uint32_t *ids;       // [64]
  float *vals;         // [64]
  uint32_t *token_out;          // optional: ids[0]
  uint32_t *token_hist;         // optional: token history [hist_cap], indexed by sp->step
  uint32_t hist_cap;
  StepParams *sp;               // optional: step counter advanced by the last CTA
  uint32_t *err;
};
int topk_blocks(uint32_t V);
cudaError_t launch_topk64(const TopkArgs &a, cudaStream_t s, bool pdl);
// Q8 LM head for B <= 64 hidden states at once (lmhead.cu)
struct LmHeadArgs {
  const uint8_t *tiles;  // Q8 tiles of the head, [V/16 row tiles][K/32]
  uint32_t row_tiles, K, V, B;
  const uint4 *xf;       // set by launch_lmhead_q8 (the token fragments)
  float *logits;         // [B][V]
  uint32_t *err;
};
size_t lmhead_frag_words(uint32_t B, uint32_t K);
// Q4 projections for B <= 64 hidden states at once (lmhead.cu): split-K partials, then an
// ordered sum with the epilogue (EPI_STORE or EPI_GELU_MUL on gate|up tiles)
struct SkinnyArgs {
  const uint8_t *tiles;  // Q4 tiles, [row_tiles][K/64]
  uint32_t row_tiles, K, B, splits, kt_per_split;
  const uint4 *xf;
  float *partial;        // [splits][B][row_tiles * 16]
  uint32_t *err;
};
uint32_t skinny_splits(uint32_t row_tiles, uint32_t K);
size_t skinny_partial_floats(uint32_t B, uint32_t row_tiles, uint32_t K);
// x_ready (B >= kSkinnyTcMinTokens only): xf already holds x's blocks (skinny_tail_kernel)
cudaError_t launch_skinny_q4(const uint8_t *tiles, uint32_t row_tiles, uint32_t K, const float *x, uint32_t ldx,
                             uint32_t B, int epi, float *y, uint32_t ldy, uint32_t *xf, float *partial, uint32_t *err,
                             cudaStream_t s, bool x_ready = false);
cudaError_t launch_lmhead_q8(const float *x, uint32_t ldx, LmHeadArgs a, uint32_t *xf, cudaStream_t s);
// the tcgen05 variant (skinny_tc.cu): partials only.  launch_skinny_q4 picks it for batches of
// kSkinnyTcMinTokens or more, where its cost (which does not grow with the batch) is below
// the mma.sync tiles' (which grows with the token groups)
constexpr uint32_t kSkinnyTcMinTokens = 17;
uint32_t skinny_tc_splits(uint32_t row_tiles, uint32_t K);
size_t skinny_tc_x_bytes(uint32_t K);
size_t skinny_tc_partial_floats(uint32_t B, uint32_t row_tiles, uint32_t K);
cudaError_t launch_skinny_q4_tc(const uint8_t *tiles, uint32_t row_tiles, uint32_t K, const float *x, uint32_t ldx,
                                uint32_t B, uint8_t *xs, float *partial, uint32_t *err, uint32_t *splits,
                                cudaStream_t s, bool x_ready = false);
// split sum + (post norm) + residual add + norm + the next GEMM's activation blocks, one
// token row per CTA (skinny_tc.cu); the batched step's o and down epilogues for 17-64 tokens
cudaError_t launch_skinny_tail(const float *partial, uint32_t splits, uint32_t B, uint32_t H, const float *post_w,
                               float *x, const float *next_w, float *y, float eps, float scalar, uint8_t *xs,
                               cudaStream_t s);
// scratch of launch_skinny_q4 and launch_lmhead_q8 for up to B tokens and K columns
size_t skinny_x_words(uint32_t B, uint32_t K);
// greedy (top-1 of the softcapped keys) of each of n rows of V logits
cudaError_t launch_argmax_rows(const float *logits, uint32_t n, uint32_t V, uint32_t *ids, cudaStream_t s);

// embedding + step advance for the device-resident decode loop
// Device copy of one DynamicRingBuffer's layer-0 slot metadata (src/ring_buffer.zig:
// 21-44): the decode step's slot lists come from layer 0 (forward.zig:44-45).
constexpr uint32_t kRingSlots = 4096, kRingRecallStart = 4096 - 128, kRingMaxBoundaries = 1024;
struct RingDevState {
  uint32_t anchors, window, nb, ingested;  // window = windowSize(0); nb = boundaries marked so far
  uint32_t next_clock, step, pad0, pad1;   // device loop: clock of its next step, steps taken
  uint32_t clocks[kRingSlots];
  uint32_t boundary[kRingMaxBoundaries];   // turn boundaries, slot i % 1024 (markBoundary)
  uint8_t active[kRingSlots];
};
struct RingStepArgs {
  RingDevState *ring = nullptr;
  uint32_t clock = 0, sliding_window = 0, chunk_len = 0;
  int activate = 0;  // activateSlot(0, clock) first
  int prev = 0;      // getPrefillPrevSlots(0, clock, chunk_len) into active_out instead
  int loop = 0;      // clock = ring->next_clock, then advance it (device loop)
  uint32_t *slot_out = nullptr, *active_out = nullptr, *n_active_out = nullptr, *sliding_out = nullptr,
           *n_sliding_out = nullptr;
  StepParams *sp = nullptr;  // also write the step's StepParams here (lists = active_out / sliding_out)
};
cudaError_t launch_ring_step(const RingStepArgs &a, cudaStream_t s);

// Sampler fields (src/sampler.zig:55-66); same layout as ch_sampler_params
struct SamplerParams {
  float temp, top_p, min_p, repeat_penalty, frequency_penalty, presence_penalty;
  uint32_t top_k;
  uint8_t suppress_thinking, suppress_critique, suppress_channel_close, reserved;
};
struct SampleArgs {
  const uint32_t *ids = nullptr;  // candidates, value descending (top-64)
  const float *vals = nullptr;
  uint32_t n = 0;
  const uint32_t *recent = nullptr;  // recent tokens (NULL: none)
  uint32_t n_recent = 0;
  uint32_t *n_recent_dev = nullptr;  // device loop: the list length lives on the device ...
  uint32_t *recent_w = nullptr;      // ... and the sampled token is appended here
  uint32_t recent_cap = 0;
  SamplerParams p{};
  uint64_t *prng = nullptr;          // [4] Xoshiro256++ state
  uint32_t *token_out = nullptr;
  const StepParams *sp = nullptr;    // device loop: history slot of the step
  uint32_t *token_hist = nullptr;
  uint32_t hist_cap = 0;
};
cudaError_t launch_sample_topk(const SampleArgs &a, cudaStream_t s);

struct StepBeginArgs {
  const uint16_t *embed;  // bf16 [V][H]
  uint32_t H;
  float embed_scale;
  const uint32_t *token;  // current token id
  float *x;               // f32 [H]
  StepParams *sp;
  const StepParams *plan; // [n_plan]
  uint32_t n_plan;
  uint32_t *err;
  const float *inv_freq_s, *inv_freq_f;  // [rot/2] each
  float2 *rope_cs;                       // out: [2][rot/2] (sliding theta, full theta)
  uint32_t rot_half;
};
cudaError_t launch_step_begin(const StepBeginArgs &a, cudaStream_t s, bool pdl);

// standalone ops (tests and prefill)
cudaError_t launch_rmsnorm_rows(const float *x, const float *w, float *y, uint32_t N, uint32_t H, float eps,
                                cudaStream_t s);
cudaError_t launch_add_rmsnorm_rows(float *x, const float *r, const float *w, float *y, uint32_t N, uint32_t H,
                                    float eps, float scalar, cudaStream_t s);
cudaError_t launch_embed_rows(const uint16_t *embed, const uint32_t *tokens, uint32_t N, uint32_t H, float scale,
                              float *x, cudaStream_t s);

// batched prefill
struct BatchQkvRopeArgs {
  const float *q, *k, *v;  // token t at q + t*q_stride, k/v + t*kv_stride
  uint32_t q_stride, kv_stride;
  const float *q_norm_w, *k_norm_w, *inv_freq;
  float *q_out;
  __half *k_cache, *v_cache;
  const uint32_t *slots;  // device
  uint32_t slot_offset, start_clock, N, nq, nkv, D, rot;
  float eps;
  int k_eq_v;
};
cudaError_t launch_batch_qkv_rope(const BatchQkvRopeArgs &a, cudaStream_t s);
struct BatchAttnArgs {
  const float *q;  // [N][nq*D] (normed + roped)
  const __half *k_cache, *v_cache;
  const uint32_t *slots;
  uint32_t N, num_prev, nq, nkv, D;
  float scale;
  int is_sliding;
  float *out;  // [N][nq*D]
};
cudaError_t launch_batch_causal_attn(const BatchAttnArgs &a, cudaStream_t s);
struct BatchGemmArgs {
  const uint8_t *tiles;  // Q4 tiles
  uint32_t M, K, N;      // rows, cols, tokens
  const float *X;        // [N][K]
  float *Y;              // EPI_STORE: [N][M]; EPI_GELU_MUL: [N][M/2]
  int epi;
};
cudaError_t launch_batch_gemm_q4(const BatchGemmArgs &a, cudaStream_t s);

// tcgen05 prefill GEMM (prefill_tc.cu).  One scratch buffer per call site:
// [16 KB split-K tile counters, zero between launches][split activation][split-K
// partials]; tc_gemm_scratch_bytes(N, M, K) bytes, 256-byte aligned, the first
// 16 KB zeroed once when it is allocated.
struct TcGemmArgs {
  const uint8_t *tiles;  // Q4 tiles [M/16][K/64]
  const uint8_t *xs;     // split activation, 16-byte aligned
  float *Y;              // EPI_STORE: [N][M]; EPI_GELU_MUL: [N][M/2]
  uint32_t M, K, N;
  int epi;
  uint32_t *err;  // device error word (bounded waits, scale range)
};
size_t tc_split_x_bytes(uint32_t N, uint32_t K);
size_t tc_gemm_scratch_bytes(uint32_t N, uint32_t M, uint32_t K);
cudaError_t launch_tc_split_x(const float *X, uint32_t N, uint32_t K, uint8_t *xs, cudaStream_t s);
// scratch_bytes: the buffer's size; a null or short buffer is refused
cudaError_t launch_batch_gemm_tc(const TcGemmArgs &a, uint8_t *scratch, size_t scratch_bytes, cudaStream_t s);
// split + GEMM: the prefill's Q4 GEMM
cudaError_t launch_batch_gemm_q4_tc(const BatchGemmArgs &g, uint8_t *scratch, size_t scratch_bytes, uint32_t *err,
                                    cudaStream_t s);

}  // namespace ch
