/*
 * channel_oracle.h -- CPU restatement of the reference's Q4 streaming-inference
 * hot path (Sullux/channel).  TEST INFRASTRUCTURE ONLY: this library is the
 * checker used by tests/, by __graft_entry__.smoke() and by bench.py's
 * cpu_baseline / --impl reference leg.  No product code path may call it.
 *
 * Parity status: pinned for the ring-buffer slot math, the greedy/penalty
 * sampler over top-k candidates and bf16 rounding (the reference's own
 * known-answer tests, ported in tests/golden/).  The Q4/Q8 matvec, GEMM,
 * attention, norm and RoPE restatements are pinned only by this restatement
 * of the reference sources (the reference has no golden vectors for them and
 * its Zig/Vulkan code cannot run here): "parity unpinned" for those rows.
 *
 * Every function cites the reference file:line it restates.  All float math is
 * IEEE f32 in program order unless stated (built with -ffp-contract=off).
 */
#ifndef CHANNEL_ORACLE_H
#define CHANNEL_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- number formats (src/tensor.zig:7-28) ---- */
uint16_t or_bf16_from_f32(float v);
float or_bf16_to_f32(uint16_t b);
uint16_t or_f16_from_f32(float v);
float or_f16_to_f32(uint16_t h);

/* ---- block quantizers (src/quant.zig:21-98) ---- */
void or_quantize_row_q4(uint32_t *dst_words, const uint16_t *src_bf16, size_t n);
void or_quantize_row_q8(uint32_t *dst_words, const uint16_t *src_bf16, size_t n);
void or_quantize_matrix(uint32_t *dst, const uint16_t *src_bf16, size_t rows, size_t cols, int mode /*4|8*/, int threads);

/* ---- seeded synthetic generators (shared spec with the CUDA generator) ---- */
uint64_t or_tensor_seed(uint64_t seed, uint32_t layer, uint32_t tensor_id);
float or_gen_normal(uint64_t tseed, uint64_t stream, uint64_t i);
void or_gen_q4_matrix(uint32_t *dst_words, size_t rows, size_t cols, uint64_t tseed, float scale_std, int threads);
void or_gen_bf16(uint16_t *dst, size_t n, uint64_t tseed, float mean, float std, int threads);
void or_gen_f32(float *dst, size_t n, uint64_t tseed, float mean, float std);

/* ---- decode matvecs (shaders/gemv_q4.wgsl, fused_qkv_q4.wgsl, fused_mlp_q4.wgsl, gemv_q8.wgsl) ---- */
void or_gemv_q4(float *y, const uint32_t *W, const float *x, size_t M, size_t K, int threads);
void or_gemv_q8(float *y, const uint32_t *W, const float *x, size_t M, size_t K, int threads);
void or_fused_mlp_q4(float *act, const uint32_t *Wg, const uint32_t *Wu, const float *x, size_t M, size_t K, int threads);
float or_gelu_tanh(float x);

/* ---- norms (src/kernels.zig:18-33, shaders/add_rmsnorm.wgsl:15-51) ---- */
void or_rmsnorm(float *y, const float *x, const float *w, size_t n, float eps);
void or_add_rmsnorm(float *x, const float *r, const float *w, float *y, size_t n, float eps, float scalar);

/* ---- qk-norm + RoPE + KV write (shaders/qkv_rope.wgsl:25-180) ----
 * q_out [nq*D]; K/V caches are f16 [slots][nkv*D]; the new K/V go to `slot`. */
void or_rope_inv_freq(float *inv_freq, uint32_t rot_dim, float theta);
void or_qkv_rope(float *q_out, uint16_t *k_cache, uint16_t *v_cache, const float *q, const float *k, const float *v,
                 const float *q_norm_w, const float *k_norm_w, uint32_t nq, uint32_t nkv, uint32_t D, uint32_t rot_dim,
                 int k_eq_v, float theta, float eps, uint32_t clock, uint32_t slot);

/* ---- decode attention (shaders/decode_attn.wgsl:24-218) ---- */
void or_decode_attn(float *out, const float *q, const uint16_t *k_cache, const uint16_t *v_cache, const uint32_t *slots,
                    uint32_t S, uint32_t nq, uint32_t nkv, uint32_t D, float scale);

/* ---- sampling (shaders/topk_pass1.wgsl:17-19, topk_pass2.wgsl; src/kernels.zig:133-143) ----
 * Top-64 of softcap(logits) sorted by value desc, ties by lowest index. */
void or_topk64(uint32_t *ids, float *vals, const float *logits, size_t V);
uint32_t or_argmax(const float *logits, size_t V);
float or_softcap(float v);
/* Sampler.sampleTopK greedy/penalty path (src/sampler.zig:210-266, temp <= 0). */
uint32_t or_sample_topk_greedy(const uint32_t *ids, const float *vals, size_t n, const uint32_t *recent, size_t n_recent,
                               float repeat_penalty, float frequency_penalty, float presence_penalty,
                               int suppress_thinking, int suppress_channel_close, int suppress_critique);
/* Zig std.Random.DefaultPrng (Xoshiro256++ seeded by SplitMix64) and Random.float(f32) */
void or_prng_seed(uint64_t *state4, uint64_t seed);
uint64_t or_prng_next(uint64_t *state4);
float or_prng_float(uint64_t *state4);
/* Sampler.sampleTopK (src/sampler.zig:217-317); params = {temp, top_p, min_p, repeat,
 * frequency, presence}; flags bit 0 suppress_thinking, 1 suppress_critique, 2
 * suppress_channel_close; recent NULL = none; advances prng by one draw when it samples */
uint32_t or_sample_topk(const uint32_t *ids, const float *vals, size_t n, const uint32_t *recent, size_t n_recent,
                        const float *params, int flags, uint64_t *prng);

/* ---- batched prefill ops (shaders/batch_*.wgsl) ---- */
void or_batch_gemm_q4(float *Y, const uint32_t *W, const float *X, size_t N, size_t M, size_t K, int threads);
void or_batch_fused_mlp_q4(float *Y, const uint32_t *Wg, const uint32_t *Wu, const float *X, size_t N, size_t M, size_t K, int threads);
void or_batch_rmsnorm(float *Y, const float *X, const float *w, size_t N, size_t H, float eps);
void or_batch_add_rmsnorm(float *X, const float *R, const float *w, float *Y, size_t N, size_t H, float eps, float scalar);
void or_batch_qkv_rope(float *q_out, uint16_t *k_cache, uint16_t *v_cache, const float *q, const float *k, const float *v,
                       const float *q_norm_w, const float *k_norm_w, uint32_t N, uint32_t nq, uint32_t nkv, uint32_t D,
                       uint32_t rot_dim, int k_eq_v, float theta, float eps, uint32_t start_clock, const uint32_t *slots,
                       uint32_t slot_offset);
void or_batch_causal_attn(float *out, const float *q, const uint16_t *k_cache, const uint16_t *v_cache, const uint32_t *slots,
                          uint32_t N, uint32_t num_prev, uint32_t nq, uint32_t nkv, uint32_t D, float scale, int is_sliding,
                          int threads);

/* ---- ring buffer (src/ring_buffer.zig:21-391), metadata only ---- */
typedef struct or_ring or_ring;
or_ring *or_ring_create(uint32_t num_layers, uint32_t num_anchors);
void or_ring_destroy(or_ring *r);
void or_ring_reset(or_ring *r);
void or_ring_set_num_anchors(or_ring *r, size_t n);
size_t or_ring_num_anchors(const or_ring *r);
size_t or_ring_total_ingested(const or_ring *r);
size_t or_ring_window_size(const or_ring *r, size_t layer);
size_t or_ring_recall_start(const or_ring *r, size_t layer);
size_t or_ring_get_slot_index(const or_ring *r, size_t layer, size_t clock);
size_t or_ring_activate_slot(or_ring *r, size_t layer, size_t clock);
void or_ring_deactivate_slot(or_ring *r, size_t layer, size_t clock);
void or_ring_rollback_clock(or_ring *r, size_t target_clock);
void or_ring_write_kv_meta(or_ring *r, size_t layer, size_t clock);
void or_ring_write_recall_meta(or_ring *r, size_t layer, size_t rank, size_t clock);
void or_ring_clear_recall(or_ring *r);
void or_ring_mark_boundary(or_ring *r, size_t clock, int span_type, float salience);
void or_ring_record_attention(or_ring *r, size_t layer, size_t slot, float mass);
float or_ring_attention_mass(const or_ring *r, size_t layer, size_t slot);
float or_ring_slot_salience(const or_ring *r, size_t slot);
float or_ring_working_set_gini(const or_ring *r);
int or_ring_is_saturated(const or_ring *r, float capacity_threshold, float gini_threshold);
size_t or_ring_evict_low_salience(or_ring *r, size_t min_clock, size_t max_clock, size_t evict_count);
int or_ring_is_active(const or_ring *r, size_t layer, size_t slot);
size_t or_ring_slot_clock(const or_ring *r, size_t layer, size_t slot);
size_t or_ring_active_slots(const or_ring *r, size_t layer, size_t clock, int is_sliding, size_t sliding_window, uint32_t *out);
size_t or_ring_prefill_prev_slots(const or_ring *r, size_t layer, size_t start_clock, size_t chunk_len, uint32_t *out);

/* ---- whole-model forward (GPU dispatch order: src/gpu/model_dispatch.zig:10-45,128-153;
 *      batched prefill: src/gpu/batch_dispatch.zig:27-172) ---- */
typedef struct {
  uint32_t vocab, hidden, inter, layers, n_q, n_kv, head_dim, rot_dim;
  float eps, theta_sliding, theta_full;
  uint32_t sliding_window;
  uint8_t layer_full[64]; /* 1 = full attention, 0 = sliding */
} or_model_cfg;

typedef struct {
  const uint32_t *wq, *wk, *wv, *wo, *wg, *wu, *wd; /* quant.zig Q4 blocks */
  const float *input_norm, *q_norm, *k_norm, *post_attn_norm, *pre_ffn_norm, *post_ffn_norm; /* post_* may be NULL */
  float layer_scalar;
} or_layer;

typedef struct or_model or_model;
or_model *or_model_create(const or_model_cfg *cfg, const or_layer *layers, const uint32_t *lm_head_q8, const float *final_norm,
                          int threads);
void or_model_destroy(or_model *m);
void or_model_reset_kv(or_model *m);
/* x: f32[hidden] (embedding row * sqrt(H)). Writes top-64 and returns ids[0]. */
uint32_t or_model_forward_token(or_model *m, const float *x, uint32_t clock, uint32_t slot, const uint32_t *active,
                                uint32_t n_active, const uint32_t *sliding, uint32_t n_sliding, uint32_t *topk_ids,
                                float *topk_vals);
/* Batched prefill; X: f32[N*hidden]; slots: prev ++ new (n_prev + N entries). */
uint32_t or_model_prefill(or_model *m, const float *X, uint32_t N, const uint32_t *slots, uint32_t start_clock,
                          uint32_t n_prev, uint32_t *topk_ids, float *topk_vals);
/* Last normed hidden state / residual (for intermediate checks). */
const float *or_model_x(const or_model *m);
const float *or_model_normed_x(const or_model *m);
const uint16_t *or_model_k_cache(const or_model *m, uint32_t layer);
const uint16_t *or_model_v_cache(const or_model *m, uint32_t layer);

/* embedding expand (src/model/forward.zig:33-37, src/gpu/batch_dispatch.zig:14-23) */
void or_embed(float *x, const uint16_t *embed_bf16, const uint32_t *tokens, size_t n, size_t H);

#ifdef __cplusplus
}
#endif
#endif
