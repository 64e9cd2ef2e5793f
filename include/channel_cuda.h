/*
 * channel_cuda.h -- C-ABI of libchannel_b200.so, the B200 (sm_100a) replacement
 * for the Vulkan GPU backend of Sullux/channel (src/gpu.zig, src/gpu/*.zig).
 *
 * Plain C types only: pointers, sizes, fixed-width integers.  Every call
 * returns an int status (CH_OK = 0, negative on error) unless noted; the
 * message of the last failure on the calling thread is ch_last_error().
 * Calls on one ch_model are not thread-safe (the reference drives its GPU
 * context from the single server thread, src/server.zig:259-281).
 *
 * Host pointers are ordinary (pageable) host memory unless the name says
 * `_dev`, in which case it is a CUDA device pointer on the context's device
 * and the call is asynchronous on the context stream (ch_ctx_stream).
 */
#ifndef CHANNEL_CUDA_H
#define CHANNEL_CUDA_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CH_API_VERSION 2

typedef enum {
  CH_OK = 0,
  CH_EINVAL = -1,   /* bad argument (shape, pointer, size)                         */
  CH_ENOMEM = -2,   /* device or host allocation failed                            */
  CH_ECUDA = -3,    /* CUDA runtime error                                          */
  CH_ETIMEOUT = -4, /* a bounded device wait gave up (status word set by a kernel) */
  CH_EBATCH = -5,   /* BatchTooLarge (src/gpu/batch_dispatch.zig:42)               */
  CH_ESTATE = -6,   /* call not valid in the current state                         */
  CH_EDEVICE = -7,  /* a kernel reported a bad slot / list entry                   */
  CH_ECOMM = -8     /* multi-GPU communicator error                                */
} ch_status;

typedef struct ch_ctx ch_ctx;
typedef struct ch_model ch_model;
typedef struct ch_ring ch_ring;

/* TopKCandidate (src/model/types.zig:115-118) */
typedef struct {
  uint32_t id;
  float val;
} ch_topk;

const char *ch_last_error(void);
int ch_api_version(void);

/* ------------------------------------------------------------------------
 * Context -- replaces GpuContext.init / deinit (src/gpu/context.zig:17-107,109)
 * ---------------------------------------------------------------------- */
int ch_ctx_create(int device, ch_ctx **out);
void ch_ctx_destroy(ch_ctx *ctx);
int ch_ctx_synchronize(ch_ctx *ctx);
void *ch_ctx_stream(ch_ctx *ctx); /* cudaStream_t */
/* Reads and clears the device status word (bit 0 bulk-copy wait timeout,
 * bit 1 bad slot, bit 2 bad slot-list entry, bit 3 peer wait timeout, bit 4 a Q4
 * block scale with |d| >= 16, outside the tensor-core GEMM's exact range). */
int ch_ctx_device_status(ch_ctx *ctx, uint32_t *flags);

/* ------------------------------------------------------------------------
 * Model -- replaces GpuModelContext.init / deinit (src/gpu/model_gpu.zig:68-216)
 * ---------------------------------------------------------------------- */
/* ModelConfig subset (src/model/types.zig:43-62) */
typedef struct {
  uint32_t vocab_size, hidden_size, intermediate_size, num_hidden_layers;
  uint32_t num_attention_heads, num_key_value_heads, head_dim, rotary_dim;
  float rms_norm_eps, rope_theta, rope_theta_full;
  uint32_t sliding_window;     /* decode sliding list length used by the caller's ring */
  uint32_t max_prefill_tokens; /* BatchPrefillContext max_tokens (model_gpu.zig:178): 1024 */
  uint8_t layer_types[64];     /* 0 = sliding_attention, 1 = full_attention (types.zig:61,109) */
} ch_model_config;

/* LayerWeights (src/model/types.zig:13-41): projections already quantized by
 * quantizeRowQ4_0 (src/quant.zig:58-98, 5 words per 32 weights), norms as f32
 * (createNormBuffer, model_gpu.zig:57-66).  post_* may be NULL. */
typedef struct {
  const uint32_t *q_proj, *k_proj, *v_proj, *o_proj, *gate_proj, *up_proj, *down_proj;
  const float *input_norm, *q_norm, *k_norm, *post_attn_norm, *pre_ffn_norm, *post_ffn_norm;
  float layer_scalar;
} ch_layer_weights;

/* Uploads and repacks every projection, the Q8_0 LM head (quantizeRowQ8_0 of
 * the tied embedding, model_gpu.zig:157) and the norms; allocates the 4,096-slot
 * f16 KV cache per layer.  embed_bf16 (vocab x hidden) is optional and enables
 * device-side embedding lookup. */
int ch_model_create(ch_ctx *ctx, const ch_model_config *cfg, const ch_layer_weights *layers, const uint32_t *lm_head_q8,
                    const float *final_norm, const uint16_t *embed_bf16, ch_model **out);
/* Same model with seeded synthetic weights generated on the device (Q4 codes
 * uniform in [-8,7], scales |N(0,0.02)| as f16, embedding bf16 N(0,0.02), LM head
 * = Q8_0 of the embedding, norms 1+N(0,0.02)); generator shared with the oracle. */
int ch_model_create_synthetic(ch_ctx *ctx, const ch_model_config *cfg, uint64_t seed, ch_model **out);

/* LayerWeights as the reference loads them from safetensors (bf16, row-major
 * [out][in], src/model/types.zig:13-41).  NULL v_proj = k_proj (attention_k_eq_v);
 * NULL input / q / k / pre-FFN norm = all ones; NULL post_attn / post_ffn norm =
 * the layer has none. */
typedef struct {
  const uint16_t *q_proj, *k_proj, *v_proj, *o_proj, *gate_proj, *up_proj, *down_proj;
  const uint16_t *input_norm, *q_norm, *k_norm, *post_attn_norm, *pre_ffn_norm, *post_ffn_norm;
  float layer_scalar;
} ch_layer_weights_bf16;
/* GpuModelContext.init with quantize-on-load (src/gpu/model_gpu.zig:44-55,68-127):
 * uploads every bf16 projection and quantizes it to Q4_0 on the device
 * (quantizeRowQ4_0, quant.zig:58-98, bit-exact), norms bf16 -> f32
 * (createNormBuffer, model_gpu.zig:57-66), the tied embedding (vocab x hidden,
 * required) to the Q8_0 LM head (model_gpu.zig:157) and the device embedding
 * table.  final_norm_bf16 NULL = all ones.  One GPU. */
int ch_model_create_bf16(ch_ctx *ctx, const ch_model_config *cfg, const ch_layer_weights_bf16 *layers,
                         const uint16_t *embed_bf16, const uint16_t *final_norm_bf16, ch_model **out);

/* Tensor-parallel decode (no counterpart in the reference, which runs one GPU):
 * shard `rank` of `world` (<= 8, one process per GPU) of the same synthetic model.
 * q|k|v and the KV cache are split by heads, o_proj / down_proj by output rows,
 * gate/up by intermediate rows, the LM head by vocab rows; norms and the embedding
 * are replicated.  Each rank's persistent decode kernel writes its output rows
 * straight into every rank's copy of the next phase's input (NVLink peer stores
 * through CUDA IPC) and all ranks meet at one arrival counter per phase, so the
 * ranks compute identical tokens.  Before decoding, every rank gets its handle
 * with ch_model_exchange_handle, the caller all-gathers the world handles in rank
 * order and every rank passes them to ch_model_attach_peers.  All ranks must then
 * make the same sequence of decode / prefill calls (prefill runs token by token
 * through the decode kernel); after ch_model_zero_state the caller synchronizes
 * the ranks before the next call.  ch_kv_read / ch_kv_write on a shard touch
 * only the rank's kv heads (see there). */
#define CH_IPC_HANDLE_BYTES 64
int ch_model_create_synthetic_sharded(ch_ctx *ctx, const ch_model_config *cfg, uint64_t seed, uint32_t rank,
                                      uint32_t world, ch_model **out);
int ch_model_exchange_handle(ch_model *m, void *handle /* CH_IPC_HANDLE_BYTES */);
int ch_model_attach_peers(ch_model *m, const void *handles /* world x CH_IPC_HANDLE_BYTES, rank order */);
void ch_model_destroy(ch_model *m);
/* Zero KV caches and decode state (src/server.zig:76-82). */
int ch_model_zero_state(ch_model *m);
/* Device pointer and logical shape of one repacked weight (which: 0 q|k|v,
 * 1 o_proj, 2 gate|up interleaved (rows = 2*intermediate), 3 down_proj,
 * 4 LM head Q8) -- for single-kernel measurement through the op-level calls. */
int ch_model_weight_tiles(ch_model *m, uint32_t layer, int which, void **tiles_dev, uint32_t *rows, uint32_t *cols);

/* ------------------------------------------------------------------------
 * Decode -- replaces gpuDispatchForwardToken (src/gpu/model_dispatch.zig:128-153)
 * x: f32[hidden] (embedding row * sqrt(hidden), forward.zig:33-37).
 * active / sliding: physical slot lists from DynamicRingBuffer.getActiveSlotsLayer
 * (layer 0, used by every layer, forward.zig:42-45).  topk_out: 64 entries or
 * NULL; token_out: greedy token (topk[0].id) or NULL.  When both are NULL the
 * logits tail is skipped (the reference's no-logits command buffer).
 * ---------------------------------------------------------------------- */
int ch_forward_token(ch_model *m, const float *x, uint32_t clock, uint32_t slot, const uint32_t *active, uint32_t n_active,
                     const uint32_t *sliding, uint32_t n_sliding, ch_topk *topk_out, uint32_t *token_out);

/* ------------------------------------------------------------------------
 * Prefill -- replaces gpuDispatchPrefillBatch (src/gpu/batch_dispatch.zig:27-172)
 * tokens: n_tokens ids (1..max_prefill_tokens, else CH_EBATCH); embed_bf16: host
 * table (NULL -> device table from model creation); slots: num_prev_slots
 * previous slots followed by the n_tokens new slots; topk_out: 64 or NULL.
 * logits_out / logits_len: the reference's logits_out slice (batch_dispatch.zig:36,
 * 168-170) -- the first logits_len raw (pre-softcap) logits of the last token,
 * logits_len <= vocab (NULL or 0: none; one GPU only).
 * progress_fn is called after every 4 layers like the reference.
 * ---------------------------------------------------------------------- */
typedef void (*ch_progress_fn)(size_t layer_idx, size_t total_layers, void *ctx);
int ch_prefill(ch_model *m, const uint32_t *tokens, uint32_t n_tokens, const uint16_t *embed_bf16, const uint32_t *slots,
               uint32_t start_clock, uint32_t num_prev_slots, ch_topk *topk_out, float *logits_out, size_t logits_len,
               ch_progress_fn progress_fn, void *progress_ctx);

/* ------------------------------------------------------------------------
 * State access -- replaces the mapped UMA buffers the reference reads/writes
 * directly (buf_x: decode.zig:13; KV: memory.zig:106-107, snapshot.zig:97-98)
 * ---------------------------------------------------------------------- */
int ch_read_x(ch_model *m, float *x);               /* residual after the last step */
int ch_read_normed_x(ch_model *m, float *normed_x); /* final-normed hidden state    */
/* k / v: kv_dim floats (all kv heads of the slot's row).  On a tensor-parallel
 * shard only the rank's kv heads [rank*n_kv/world, (rank+1)*n_kv/world) are read
 * (the rest of k / v is left as it was) or written: the full row is every rank's
 * call over the same row. */
int ch_kv_read(ch_model *m, uint32_t layer, uint32_t slot, float *k, float *v);
int ch_kv_write(ch_model *m, uint32_t layer, uint32_t slot, const float *k, const float *v);

/* ------------------------------------------------------------------------
 * Device-resident greedy decode loop (no host round trip per token): the
 * per-step ring lists are uploaded once, then each step embeds the previous
 * token on the device and feeds its greedy token to the next step.
 * ---------------------------------------------------------------------- */
typedef struct {
  uint32_t clock, slot, n_active, n_sliding;
  const uint32_t *active, *sliding; /* host lists */
} ch_step_desc;
int ch_decode_plan(ch_model *m, const ch_step_desc *steps, uint32_t n_steps); /* requires the device embedding */
int ch_decode_run(ch_model *m, uint32_t first_token, uint32_t n_steps);     /* async; restarts at plan step 0 */
int ch_decode_continue(ch_model *m, uint32_t n_steps);                      /* async; next planned steps   */
int ch_decode_tokens(ch_model *m, uint32_t *tokens, uint32_t n);            /* syncs, copies step tokens */

/* ------------------------------------------------------------------------
 * Stochastic sampling on the device -- Sampler.sampleTopK (src/sampler.zig:217-317)
 * over the top-64: suppressed ids dropped, repeat / frequency / presence penalties
 * of the recent tokens with a stable re-sort, temperature softmax, min-p, top-p and
 * one draw from Zig's std.Random.DefaultPrng (Xoshiro256++ seeded by SplitMix64,
 * Random.float(f32)).  Field order and defaults as Sampler (sampler.zig:55-82).
 * ---------------------------------------------------------------------- */
typedef struct {
  float temp, top_p, min_p, repeat_penalty, frequency_penalty, presence_penalty;
  uint32_t top_k; /* kept for layout; sampleTopK uses the 64 candidates it gets */
  uint8_t suppress_thinking, suppress_critique, suppress_channel_close, reserved;
} ch_sampler_params;
typedef struct ch_sampler ch_sampler;
/* Sampler.init(seed, ...): the generator state and a device list of recent tokens
 * (capacity recent_cap) for device loops */
int ch_sampler_create(ch_ctx *ctx, const ch_sampler_params *params, uint64_t seed, uint32_t recent_cap,
                      ch_sampler **out);
void ch_sampler_destroy(ch_sampler *s);
/* replace the sampler's recent-token list (the response so far, server/decode.zig:40-60);
 * a device loop then appends every token it samples */
int ch_sampler_set_recent(ch_sampler *s, const uint32_t *recent, uint32_t n);
/* sampleTopK of n (<= 64) device candidates -> *token_dev; recent_dev NULL = no recent
 * tokens; asynchronous on the context stream (one generator draw when it samples) */
int ch_sampler_sample_topk(ch_sampler *s, const uint32_t *ids_dev, const float *vals_dev, uint32_t n,
                           const uint32_t *recent_dev, uint32_t n_recent, uint32_t *token_dev);
/* device loops of m (ch_decode_run / _continue / _run_ring) sample every step's token
 * with s and its recent list instead of taking the greedy one; NULL = greedy */
int ch_model_set_sampler(ch_model *m, ch_sampler *s);

/* ------------------------------------------------------------------------
 * Multi-stream greedy decode (no reference counterpart: the
 * reference serves one stream, src/server_queue.zig:9-145, src/server.zig:259-281).
 * Each stream owns a 4,096-slot KV cache per layer; its ring bookkeeping stays on
 * the host (ch_ring_*), one ring per stream.  A step takes one token from each of
 * up to max_batch (<= 64) distinct streams and returns each stream's greedy next token; the
 * weights are read once per step for the whole batch.  One GPU (no tensor parallel);
 * needs the device embedding.
 * ---------------------------------------------------------------------- */
typedef struct {
  uint32_t stream, token, clock, slot; /* token: the stream's current input token */
  const uint32_t *active, *sliding;    /* host lists, like ch_forward_token */
  uint32_t n_active, n_sliding;
} ch_stream_step;
int ch_streams_init(ch_model *m, uint32_t n_streams, uint32_t max_batch);
/* ch_prefill into the stream's cache; *token_out = greedy token after the prompt */
int ch_stream_prefill(ch_model *m, uint32_t stream, const uint32_t *tokens, uint32_t n_tokens, const uint32_t *slots,
                      uint32_t start_clock, uint32_t num_prev_slots, uint32_t *token_out);
int ch_streams_decode(ch_model *m, const ch_stream_step *steps, uint32_t n, uint32_t *tokens_out);
/* State of the last ch_streams_decode step (its first n entries, in step order):
 * the final-normed hidden state each token's LM head read (n x hidden) and the raw
 * pre-softcap logits (n x vocab) -- the multi-stream counterpart of ch_read_normed_x
 * and of the reference's buf_logits read (batch_dispatch.zig:168-170). */
int ch_streams_read_normed_x(ch_model *m, uint32_t n, float *normed_x);
int ch_streams_read_logits(ch_model *m, uint32_t n, float *logits);

/* ------------------------------------------------------------------------
 * Op-level entry points (device pointers, async on the context stream).
 * Weight tiles: 16 rows x 64 k (Q4) / 16 x 32 (Q8), 576 bytes each.
 * ---------------------------------------------------------------------- */
size_t ch_q4_tile_bytes(uint32_t rows, uint32_t cols);
size_t ch_q8_tile_bytes(uint32_t rows, uint32_t cols);
/* quant.zig Q4 blocks (rows x cols/32 x 5 words) -> tiles; rows % 16, cols % 64 */
int ch_q4_pack(ch_ctx *ctx, const uint32_t *blocks_dev, uint32_t rows, uint32_t cols, void *tiles_dev);
/* gate/up pair (rows each) -> interleaved tiles for ch_fused_mlp_q4 (2*rows rows) */
int ch_q4_pack_gateup(ch_ctx *ctx, const uint32_t *gate_dev, const uint32_t *up_dev, uint32_t rows, uint32_t cols,
                      void *tiles_dev);
/* Q8_0 blocks (rows x cols/32 x 9 words) -> tiles */
int ch_q8_pack(ch_ctx *ctx, const uint32_t *blocks_dev, uint32_t rows, uint32_t cols, void *tiles_dev);
/* gemv_q4.wgsl: y[rows] = W x */
int ch_gemv_q4(ch_ctx *ctx, const void *tiles_dev, uint32_t rows, uint32_t cols, const float *x_dev, float *y_dev);
/* fused_mlp_q4.wgsl: act[rows] = gelu_tanh(Wg x) * (Wu x) */
int ch_fused_mlp_q4(ch_ctx *ctx, const void *gateup_tiles_dev, uint32_t rows, uint32_t cols, const float *x_dev,
                    float *act_dev);
/* gemv_q8.wgsl */
int ch_gemv_q8(ch_ctx *ctx, const void *tiles_dev, uint32_t rows, uint32_t cols, const float *x_dev, float *y_dev);
/* No counterpart in the reference.  ch_gemv_q4 without a context and without
 * allocating: for callers that may not allocate device memory -- a host
 * runtime whose pool allocator owns the device's memory, a serving loop that
 * bans cudaFree (it synchronizes the device) once it is running, or a binding
 * that may only use the buffers its caller hands over.  The stream-K scratch
 * lives in one static device array of about 300 KB that every GPU loading the
 * library holds until exit.  Limits: rows <= 32768, cols <= 16384 (CH_EINVAL
 * beyond).  Runs on the current device, asynchronously on `stream` (a
 * cudaStream_t; NULL = default stream).  The first call on a device resolves
 * the array's device address (and may load the library's CUDA module), so
 * make it once during set-up, before any stream capture.  All calls on a
 * device share the array: calls that overlap on the GPU (other streams, other
 * threads) race and must be serialized by the caller.  The call clears the
 * per-row-tile counters it uses before the kernel runs.  status_dev, if not
 * NULL, is a device word into which the kernel ORs bit 0 when a weight copy
 * stalls (the bits of ch_ctx_device_status; y is then incomplete); NULL
 * discards them. */
int ch_gemv_q4_noalloc(const void *tiles_dev, uint32_t rows, uint32_t cols, const float *x_dev, float *y_dev,
                       uint32_t *status_dev, void *stream);
/* rmsnorm.wgsl / add_rmsnorm.wgsl over n_rows rows of h */
int ch_rmsnorm(ch_ctx *ctx, const float *x_dev, const float *w_dev, float *y_dev, uint32_t n_rows, uint32_t h, float eps);
int ch_add_rmsnorm(ch_ctx *ctx, float *x_dev, const float *r_dev, const float *w_dev, float *y_dev, uint32_t n_rows,
                   uint32_t h, float eps, float scalar);
/* qkv_rope.wgsl + decode_attn.wgsl for one layer: qkv_dev = q|k|v raw
 * projections; K/V caches f16 [4096][nkv*head_dim]; the new K/V go to `slot`. */
int ch_decode_attention(ch_ctx *ctx, const float *qkv_dev, const float *q_norm_dev, const float *k_norm_dev,
                        void *k_cache_dev, void *v_cache_dev, const uint32_t *slots_dev, uint32_t n_slots, uint32_t clock,
                        uint32_t slot, uint32_t nq, uint32_t nkv, uint32_t head_dim, uint32_t rotary_dim, float theta,
                        float eps, float scale, float *out_dev);
/* batch_causal_attn.wgsl (25-223): q_dev = n_tokens x nq x head_dim (normed and roped),
 * K/V caches f16 [4096][nkv*head_dim]; token t attends to slots_dev[0 .. num_prev+t+1),
 * on a sliding layer (is_sliding) to the last 1,024 of them (:53); out_dev like q_dev.
 * Pairs of q heads per kv head run on the tensor cores (mma.sync, f32 accumulate). */
int ch_batch_causal_attention(ch_ctx *ctx, const float *q_dev, const void *k_cache_dev, const void *v_cache_dev,
                              const uint32_t *slots_dev, uint32_t n_tokens, uint32_t num_prev, uint32_t nq,
                              uint32_t nkv, uint32_t head_dim, float scale, int is_sliding, float *out_dev);
/* topk_pass1/2.wgsl: softcap + top-64, value desc then lowest index */
int ch_topk64(ch_ctx *ctx, const float *logits_dev, uint32_t vocab, uint32_t *ids_dev, float *vals_dev);
/* batch_gemm_q4.wgsl (Y[t*rows + r]) and batch_fused_mlp_q4.wgsl on tiles, on the
 * tcgen05 tensor cores: each weight (q-8)*d enters exactly as two f16 operands
 * (d split into its top 8 significant bits and the rest), the activation as an
 * f16 hi + lo pair, f32 accumulation.  The context keeps a scratch buffer (the
 * split activation, about 4 * n * cols bytes, plus split-K partials for short row
 * counts), grown on first use of a larger shape. */
int ch_batch_gemm_q4(ch_ctx *ctx, const void *tiles_dev, uint32_t rows, uint32_t cols, const float *x_dev,
                     uint32_t n_tokens, float *y_dev);
int ch_batch_fused_mlp_q4(ch_ctx *ctx, const void *gateup_tiles_dev, uint32_t rows, uint32_t cols, const float *x_dev,
                          uint32_t n_tokens, float *act_dev);
/* The same two GEMMs on the legacy mma.sync tensor path (no counterpart in the
 * reference): kept as the measured baseline of the tcgen05 kernels. */
int ch_batch_gemm_q4_mma(ch_ctx *ctx, const void *tiles_dev, uint32_t rows, uint32_t cols, const float *x_dev,
                         uint32_t n_tokens, float *y_dev);
int ch_batch_fused_mlp_q4_mma(ch_ctx *ctx, const void *gateup_tiles_dev, uint32_t rows, uint32_t cols,
                              const float *x_dev, uint32_t n_tokens, float *act_dev);
/* seeded generators (same spec as the oracle) */
int ch_gen_q4_blocks(ch_ctx *ctx, uint32_t *blocks_dev, uint32_t rows, uint32_t cols, uint64_t tensor_seed,
                     float scale_std);
int ch_gen_bf16(ch_ctx *ctx, uint16_t *dst_dev, size_t n, uint64_t tensor_seed, float mean, float std);
int ch_quantize_q8_rows(ch_ctx *ctx, const uint16_t *src_bf16_dev, uint32_t rows, uint32_t cols, uint32_t *dst_dev);
int ch_quantize_q4_rows(ch_ctx *ctx, const uint16_t *src_bf16_dev, uint32_t rows, uint32_t cols, uint32_t *dst_dev);
uint64_t ch_tensor_seed(uint64_t seed, uint32_t layer, uint32_t tensor_id);

/* ------------------------------------------------------------------------
 * Ring buffer slot math -- DynamicRingBuffer (src/ring_buffer.zig:21-391),
 * metadata only (the K/V rows live in the model's device cache).
 * ---------------------------------------------------------------------- */
ch_ring *ch_ring_create(uint32_t num_layers, uint32_t num_anchors);
void ch_ring_destroy(ch_ring *r);
void ch_ring_reset(ch_ring *r);
void ch_ring_set_num_anchors(ch_ring *r, size_t n);
size_t ch_ring_num_anchors(const ch_ring *r);
size_t ch_ring_total_ingested(const ch_ring *r);
size_t ch_ring_window_size(const ch_ring *r, size_t layer);
size_t ch_ring_get_slot_index(const ch_ring *r, size_t layer, size_t clock);
size_t ch_ring_activate_slot(ch_ring *r, size_t layer, size_t clock);
/* no reference counterpart: ch_ring_activate_slot of clocks [clock0, clock0 + n) in every
 * layer, in clock order, with each clock's layer-0 slot in slots_out (may be NULL) -- the
 * host bookkeeping of a prompt chunk in one call */
void ch_ring_activate_range(ch_ring *r, size_t clock0, size_t n, uint32_t *slots_out);
/* no reference counterpart: one ch_streams_decode step's host work for n streams, each
 * with its own ring -- ch_ring_activate_slot(rings[b], 0, clocks[b]), then the slot index
 * and the full and sliding lists of layer 0 at that clock -- written into steps[b]
 * (stream, token, clock, slot, lists) with the lists stored at lists + b * 8192 (active,
 * then sliding; the caller keeps the storage alive for the step) */
void ch_rings_fill_steps(ch_ring *const *rings, const uint32_t *streams, const uint32_t *tokens, const uint32_t *clocks,
                         uint32_t n, size_t sliding_window, ch_stream_step *steps, uint32_t *lists);
void ch_ring_deactivate_slot(ch_ring *r, size_t layer, size_t clock);
void ch_ring_rollback_clock(ch_ring *r, size_t target_clock);
void ch_ring_write_kv_meta(ch_ring *r, size_t layer, size_t clock);
void ch_ring_write_recall_meta(ch_ring *r, size_t layer, size_t rank, size_t clock);
void ch_ring_clear_recall(ch_ring *r);
void ch_ring_mark_boundary(ch_ring *r, size_t clock, int span_type, float salience);
int ch_ring_is_active(const ch_ring *r, size_t layer, size_t slot);
size_t ch_ring_slot_clock(const ch_ring *r, size_t layer, size_t slot);
size_t ch_ring_active_slots(const ch_ring *r, size_t layer, size_t clock, int is_sliding, size_t sliding_window,
                            uint32_t *out);
size_t ch_ring_prefill_prev_slots(const ch_ring *r, size_t layer, size_t start_clock, size_t chunk_len, uint32_t *out);

/* ------------------------------------------------------------------------
 * Ring lists on the device (no reference counterpart: the reference builds the
 * lists on the host every token, src/ring_buffer.zig:287-380 via forward.zig:44-45,
 * and uploads them, model_dispatch.zig:133-135).  A ch_ring_dev is a device copy of
 * a ring's layer-0 metadata (active flags, slot clocks, anchors, turn boundaries);
 * its lists are the host ring's, bit for bit, in the same order.
 * ---------------------------------------------------------------------- */
typedef struct ch_ring_dev ch_ring_dev;
int ch_ring_dev_create(ch_ctx *ctx, ch_ring_dev **out);
void ch_ring_dev_destroy(ch_ring_dev *r);
/* copy the host ring's layer-0 metadata to the device (synchronous) */
int ch_ring_dev_upload(ch_ring_dev *r, const ch_ring *host);
/* [activateSlot(0, clock) if activate, then] slotIndex(clock) -> *slot_dev (may be NULL),
 * getActiveSlotsLayer(0, clock, false, .) -> active_dev[*n_active_dev] and
 * getActiveSlotsLayer(0, clock, true, sliding_window) -> sliding_dev[*n_sliding_dev];
 * lists hold up to 4096 entries; asynchronous on the context stream */
int ch_ring_dev_lists(ch_ring_dev *r, uint32_t clock, int activate, size_t sliding_window, uint32_t *slot_dev,
                      uint32_t *active_dev, uint32_t *n_active_dev, uint32_t *sliding_dev, uint32_t *n_sliding_dev);
/* getPrefillPrevSlots(0, start_clock, chunk_len) -> out_dev[*n_dev]; asynchronous */
int ch_ring_dev_prefill_prev(ch_ring_dev *r, uint32_t start_clock, uint32_t chunk_len, uint32_t *out_dev,
                             uint32_t *n_dev);
/* Device-resident greedy loop like ch_decode_run, but every step activates its slot
 * in the device ring and builds its own lists there (clocks first_clock ..
 * first_clock + n_steps - 1): no plan, nothing uploaded per token.  r must hold the
 * host ring's state (ch_ring_dev_upload); the host ring `host` (may be NULL) gets
 * the same activations when the call returns.  Asynchronous; ch_decode_tokens
 * reads the tokens.  Afterwards ch_decode_run / ch_decode_continue need a new
 * ch_decode_plan. */
int ch_decode_run_ring(ch_model *m, ch_ring_dev *r, ch_ring *host, uint32_t first_token, uint32_t first_clock,
                       uint32_t n_steps);

#ifdef __cplusplus
}
#endif
#endif /* CHANNEL_CUDA_H */
