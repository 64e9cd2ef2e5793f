// channel_oracle.cpp -- CPU restatement of the reference hot path.  TEST
// INFRASTRUCTURE ONLY (the checker): see channel_oracle.h for the parity status.
// Built with -O2 -ffp-contract=off so every f32 expression rounds like the
// reference's scalar code.  Multithreaded by row chunks like gemvParallel
// (src/kernels.zig:53-68).
#include "channel_oracle.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <thread>
#include <vector>

// ----------------------------------------------------------------------------
// threading helper: rows [0,n) split into `threads` contiguous chunks
static void parallel_rows(size_t n, int threads, const std::function<void(size_t, size_t)> &fn) {
  if (threads <= 1 || n < 64) {
    fn(0, n);
    return;
  }
  size_t t = (size_t)threads;
  if (t > n) t = n;
  std::vector<std::thread> pool;
  size_t chunk = (n + t - 1) / t;
  for (size_t i = 0; i < t; i++) {
    size_t b = i * chunk, e = std::min(n, b + chunk);
    if (b >= e) break;
    pool.emplace_back(fn, b, e);
  }
  for (auto &th : pool) th.join();
}

static inline uint32_t fbits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
static inline float bitsf(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

// ----------------------------------------------------------------------------
// number formats -- src/tensor.zig:7-28
extern "C" uint16_t or_bf16_from_f32(float v) {
  // tensor.zig:7-13: round to nearest even by adding 0x7FFF + lsb, truncate.
  uint32_t u = fbits(v);
  uint32_t bias = 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)((u + bias) >> 16);
}
extern "C" float or_bf16_to_f32(uint16_t b) { return bitsf((uint32_t)b << 16); }

// IEEE binary16, round to nearest even (Zig @floatCast f32 -> f16).
extern "C" uint16_t or_f16_from_f32(float f) {
  uint32_t x = fbits(f);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return (uint16_t)(sign | (ax > 0x7f800000u ? 0x7e00u : 0x7c00u));
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
  if (ax >= 0x38800000u) {
    uint32_t mant = ax & 0x7fffffu;
    uint32_t e = (ax >> 23) - 127 + 15;
    uint32_t h = (e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
  }
  if (ax < 0x33000000u) return (uint16_t)sign;
  uint32_t mant = (ax & 0x7fffffu) | 0x800000u;
  int e = (int)(ax >> 23) - 127;
  int shift = -(e + 1);
  uint32_t h = mant >> shift;
  uint32_t rem = mant & ((1u << shift) - 1u);
  uint32_t half = 1u << (shift - 1);
  if (rem > half || (rem == half && (h & 1u))) h++;
  return (uint16_t)(sign | h);
}
extern "C" float or_f16_to_f32(uint16_t h) {
  uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  if (e == 0) {
    float v = (float)m * 5.9604644775390625e-08f;  // 2^-24, exact
    return sign ? -v : v;
  }
  if (e == 31) return bitsf(sign | 0x7f800000u | (m << 13));
  return bitsf(sign | ((e - 15 + 127) << 23) | (m << 13));
}

// ----------------------------------------------------------------------------
// quantizers -- src/quant.zig:21-52 (Q8_0) and :58-98 (Q4)
extern "C" void or_quantize_row_q8(uint32_t *dst, const uint16_t *src, size_t n) {
  size_t nb = n / 32;
  for (size_t b = 0; b < nb; b++) {
    float vals[32];
    float amax = 0.0f;
    for (int i = 0; i < 32; i++) {
      float v = or_bf16_to_f32(src[b * 32 + i]);
      vals[i] = v;
      float a = fabsf(v);
      if (a > amax) amax = a;
    }
    float d = amax / 127.0f;
    float id = (amax > 0.0f) ? 127.0f / amax : 0.0f;
    uint32_t *blk = dst + b * 9;
    blk[0] = fbits(d);
    uint8_t bytes[32];
    for (int i = 0; i < 32; i++) {
      int q = (int)roundf(vals[i] * id);  // std.math.round: half away from zero
      q = std::min(127, std::max(-128, q));
      bytes[i] = (uint8_t)(int8_t)q;
    }
    for (int w = 0; w < 8; w++)
      blk[1 + w] = (uint32_t)bytes[w * 4] | ((uint32_t)bytes[w * 4 + 1] << 8) | ((uint32_t)bytes[w * 4 + 2] << 16) |
                   ((uint32_t)bytes[w * 4 + 3] << 24);
  }
}

extern "C" void or_quantize_row_q4(uint32_t *dst, const uint16_t *src, size_t n) {
  size_t nb = n / 32;
  for (size_t b = 0; b < nb; b++) {
    float vals[32];
    float amax = 0.0f;
    for (int i = 0; i < 32; i++) {
      float v = or_bf16_to_f32(src[b * 32 + i]);
      vals[i] = v;
      float a = fabsf(v);
      if (a > amax) amax = a;
    }
    float d = amax / 8.0f;
    float id = (d > 0.0f) ? 1.0f / d : 0.0f;
    uint16_t s16 = or_f16_from_f32(d);
    uint16_t m16 = or_f16_from_f32(-8.0f * d);
    uint32_t *blk = dst + b * 5;
    blk[0] = (uint32_t)s16 | ((uint32_t)m16 << 16);
    uint8_t nib[32];
    for (int i = 0; i < 32; i++) {
      float t = vals[i] * id;
      t = t + 8.0f;
      int q = (int)roundf(t);
      nib[i] = (uint8_t)std::min(15, std::max(0, q));
    }
    for (int w = 0; w < 4; w++) {
      uint32_t word = 0;
      for (int k = 0; k < 8; k++) word |= (uint32_t)nib[w * 8 + k] << (4 * k);
      blk[1 + w] = word;
    }
  }
}

// quant.zig:100-170 (row-chunked; results are per-row so threading is exact)
extern "C" void or_quantize_matrix(uint32_t *dst, const uint16_t *src, size_t rows, size_t cols, int mode, int threads) {
  size_t row_words = (cols / 32) * (mode == 8 ? 9 : 5);
  parallel_rows(rows, threads, [&](size_t b, size_t e) {
    for (size_t r = b; r < e; r++) {
      if (mode == 8)
        or_quantize_row_q8(dst + r * row_words, src + r * cols, cols);
      else
        or_quantize_row_q4(dst + r * row_words, src + r * cols, cols);
    }
  });
}

// ----------------------------------------------------------------------------
// seeded synthetic generator.  Counter-based (splitmix64 finaliser) so that the
// CUDA generator produces bit-identical tensors.  N(0,1) is approximated by the
// Irwin-Hall sum of twelve 21-bit uniforms (integer sum, one exact-to-float
// conversion), so no libm call is involved and host/device agree bit for bit.
static inline uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
static inline uint64_t hash3(uint64_t tseed, uint64_t stream, uint64_t i) {
  return mix64(mix64(tseed ^ (stream * 0xD6E8FEB86659FD93ull)) ^ (i * 0xD1B54A32D192ED03ull));
}
extern "C" uint64_t or_tensor_seed(uint64_t seed, uint32_t layer, uint32_t tensor_id) {
  return mix64(mix64(seed) ^ (((uint64_t)layer << 16) | tensor_id));
}
extern "C" float or_gen_normal(uint64_t tseed, uint64_t stream, uint64_t i) {
  int64_t s = 0;
  for (int j = 0; j < 4; j++) {
    uint64_t r = hash3(tseed, stream, i * 4 + j);
    s += (int64_t)(r & 0x1FFFFF) + (int64_t)((r >> 21) & 0x1FFFFF) + (int64_t)((r >> 42) & 0x1FFFFF);
  }
  int32_t c = (int32_t)(2 * s - 12 * (int64_t)0x1FFFFF);  // |c| < 2^26: exact in int, RN to float
  return (float)c * 2.384185791015625e-07f;                // * 2^-22
}
extern "C" void or_gen_q4_matrix(uint32_t *dst, size_t rows, size_t cols, uint64_t tseed, float scale_std, int threads) {
  size_t nb = cols / 32;
  parallel_rows(rows, threads, [&](size_t b, size_t e) {
    for (size_t r = b; r < e; r++)
      for (size_t j = 0; j < nb; j++) {
        uint64_t blk = r * nb + j;
        uint64_t ha = hash3(tseed, 0, blk * 2), hb = hash3(tseed, 0, blk * 2 + 1);
        float z = or_gen_normal(tseed, 1, blk);
        float d = fabsf(z) * scale_std;
        uint16_t d16 = or_f16_from_f32(d);
        uint16_t m16 = or_f16_from_f32(-8.0f * or_f16_to_f32(d16));
        uint32_t *o = dst + blk * 5;
        o[0] = (uint32_t)d16 | ((uint32_t)m16 << 16);
        o[1] = (uint32_t)ha;
        o[2] = (uint32_t)(ha >> 32);
        o[3] = (uint32_t)hb;
        o[4] = (uint32_t)(hb >> 32);
      }
  });
}
extern "C" void or_gen_bf16(uint16_t *dst, size_t n, uint64_t tseed, float mean, float std, int threads) {
  parallel_rows(n, threads, [&](size_t b, size_t e) {
    for (size_t i = b; i < e; i++) {
      float z = or_gen_normal(tseed, 2, i);
      float v = mean + z * std;
      dst[i] = or_bf16_from_f32(v);
    }
  });
}
extern "C" void or_gen_f32(float *dst, size_t n, uint64_t tseed, float mean, float std) {
  for (size_t i = 0; i < n; i++) {
    float z = or_gen_normal(tseed, 3, i);
    dst[i] = mean + z * std;
  }
}

// ----------------------------------------------------------------------------
// Q4 / Q8 matvec -- shaders/gemv_q4.wgsl:15-26,44-72; gemv_q8.wgsl:41-63
static inline float unpack_dot2(uint32_t w, const float *xa) {
  // gemv_q4.wgsl:15-26: (q - 8) * x for 8 nibbles, little nibble first
  float n0 = (float)(w & 0xFu) - 8.0f, n1 = (float)((w >> 4) & 0xFu) - 8.0f;
  float n2 = (float)((w >> 8) & 0xFu) - 8.0f, n3 = (float)((w >> 12) & 0xFu) - 8.0f;
  float n4 = (float)((w >> 16) & 0xFu) - 8.0f, n5 = (float)((w >> 20) & 0xFu) - 8.0f;
  float n6 = (float)((w >> 24) & 0xFu) - 8.0f, n7 = (float)(w >> 28) - 8.0f;
  return n0 * xa[0] + n1 * xa[1] + n2 * xa[2] + n3 * xa[3] + n4 * xa[4] + n5 * xa[5] + n6 * xa[6] + n7 * xa[7];
}
static inline float q4_row_dot(const uint32_t *row, const float *x, size_t nb) {
  float acc = 0.0f;
  for (size_t b = 0; b < nb; b++) {
    const uint32_t *blk = row + b * 5;
    float s = or_f16_to_f32((uint16_t)(blk[0] & 0xFFFFu));  // unpack2x16float(W[blk]).x; `min` ignored
    const float *xb = x + b * 32;
    float dot = unpack_dot2(blk[1], xb) + unpack_dot2(blk[2], xb + 8) + unpack_dot2(blk[3], xb + 16) +
                unpack_dot2(blk[4], xb + 24);
    acc += s * dot;
  }
  return acc;
}
extern "C" void or_gemv_q4(float *y, const uint32_t *W, const float *x, size_t M, size_t K, int threads) {
  size_t nb = K / 32;
  parallel_rows(M, threads, [&](size_t b, size_t e) {
    for (size_t r = b; r < e; r++) y[r] = q4_row_dot(W + r * nb * 5, x, nb);
  });
}
static inline float q8_row_dot(const uint32_t *row, const float *x, size_t nb) {
  float acc = 0.0f;
  for (size_t b = 0; b < nb; b++) {
    const uint32_t *blk = row + b * 9;
    float s = bitsf(blk[0]);
    const float *xb = x + b * 32;
    for (int p = 0; p < 4; p++) {  // gemv_q8.wgsl: 8 int8 per lane, s * sum_wx
      uint32_t wa = blk[1 + 2 * p], wb = blk[2 + 2 * p];
      float sum = 0.0f;
      for (int i = 0; i < 4; i++) sum += (float)(int8_t)((wa >> (8 * i)) & 0xFFu) * xb[p * 8 + i];
      for (int i = 0; i < 4; i++) sum += (float)(int8_t)((wb >> (8 * i)) & 0xFFu) * xb[p * 8 + 4 + i];
      acc += s * sum;
    }
  }
  return acc;
}
extern "C" void or_gemv_q8(float *y, const uint32_t *W, const float *x, size_t M, size_t K, int threads) {
  size_t nb = K / 32;
  parallel_rows(M, threads, [&](size_t b, size_t e) {
    for (size_t r = b; r < e; r++) y[r] = q8_row_dot(W + r * nb * 9, x, nb);
  });
}
// src/kernels.zig:7-10 (same constants in fused_mlp_q4.wgsl:15-18)
extern "C" float or_gelu_tanh(float x) {
  float inner = 0.7978845608f * (x + 0.044715f * x * x * x);
  return 0.5f * x * (1.0f + tanhf(inner));
}
// shaders/fused_mlp_q4.wgsl:33-128: act = gelu_tanh(Wg x) * (Wu x)
extern "C" void or_fused_mlp_q4(float *act, const uint32_t *Wg, const uint32_t *Wu, const float *x, size_t M, size_t K,
                                int threads) {
  size_t nb = K / 32;
  parallel_rows(M, threads, [&](size_t b, size_t e) {
    for (size_t r = b; r < e; r++) {
      float g = q4_row_dot(Wg + r * nb * 5, x, nb);
      float u = q4_row_dot(Wu + r * nb * 5, x, nb);
      act[r] = or_gelu_tanh(g) * u;
    }
  });
}

// ----------------------------------------------------------------------------
// norms -- src/kernels.zig:18-26 (rmsNorm), shaders/add_rmsnorm.wgsl:15-51
extern "C" void or_rmsnorm(float *y, const float *x, const float *w, size_t n, float eps) {
  float ss = 0.0f;
  for (size_t i = 0; i < n; i++) ss += x[i] * x[i];
  float inv = 1.0f / sqrtf(ss / (float)n + eps);
  for (size_t i = 0; i < n; i++) y[i] = x[i] * inv * w[i];
}
extern "C" void or_add_rmsnorm(float *x, const float *r, const float *w, float *y, size_t n, float eps, float scalar) {
  float ss = 0.0f;
  for (size_t i = 0; i < n; i++) {
    float v = (x[i] + r[i]) * scalar;
    x[i] = v;
    ss += v * v;
  }
  float inv = 1.0f / sqrtf(ss / (float)n + eps);
  for (size_t i = 0; i < n; i++) y[i] = x[i] * inv * w[i];
}

// ----------------------------------------------------------------------------
// RoPE -- src/kernels.zig:101-119, shaders/qkv_rope.wgsl:63-83.
// inv_freq[i] = 1 / theta^(2i/rot) and cos/sin(angle) are evaluated in double and
// rounded once to f32 (a correctly rounded restatement of the f32 expressions).
extern "C" void or_rope_inv_freq(float *inv_freq, uint32_t rot_dim, float theta) {
  for (uint32_t i = 0; i < rot_dim / 2; i++) {
    float e = (2.0f * (float)i) / (float)rot_dim;
    inv_freq[i] = (float)(1.0 / pow((double)theta, (double)e));
  }
}
static void rope_head_norm(float *out, const float *in, const float *w, uint32_t D, uint32_t rot, const float *inv_freq,
                           uint32_t clock, float eps) {
  float ss = 0.0f;
  for (uint32_t d = 0; d < D; d++) ss += in[d] * in[d];
  float inv = 1.0f / sqrtf(ss / (float)D + eps);
  uint32_t half = rot / 2;
  for (uint32_t d = 0; d < half; d++) {
    float v0 = in[d] * inv * w[d];
    float v1 = in[d + half] * inv * w[d + half];
    float ang = (float)clock * inv_freq[d];
    float c = (float)cos((double)ang), s = (float)sin((double)ang);
    out[d] = v0 * c - v1 * s;
    out[d + half] = v0 * s + v1 * c;
  }
  for (uint32_t d = rot; d < D; d++) out[d] = in[d] * inv * w[d];
}
static void unit_norm(float *out, const float *in, uint32_t D, float eps) {
  float ss = 0.0f;
  for (uint32_t d = 0; d < D; d++) ss += in[d] * in[d];
  float inv = 1.0f / sqrtf(ss / (float)D + eps);
  for (uint32_t d = 0; d < D; d++) out[d] = in[d] * inv;
}
static void qkv_rope_token(float *q_out, uint16_t *kc, uint16_t *vc, const float *q, const float *k, const float *v,
                           const float *qw, const float *kw, uint32_t nq, uint32_t nkv, uint32_t D, uint32_t rot,
                           int k_eq_v, const float *inv_freq, float eps, uint32_t clock, uint32_t slot) {
  std::vector<float> tmp(D);
  for (uint32_t h = 0; h < nq; h++) rope_head_norm(q_out + h * D, q + h * D, qw, D, rot, inv_freq, clock, eps);
  size_t kv_dim = (size_t)nkv * D;
  for (uint32_t h = 0; h < nkv; h++) {
    rope_head_norm(tmp.data(), k + h * D, kw, D, rot, inv_freq, clock, eps);
    for (uint32_t d = 0; d < D; d++) kc[(size_t)slot * kv_dim + h * D + d] = or_f16_from_f32(tmp[d]);
    unit_norm(tmp.data(), (k_eq_v ? k : v) + h * D, D, eps);
    for (uint32_t d = 0; d < D; d++) vc[(size_t)slot * kv_dim + h * D + d] = or_f16_from_f32(tmp[d]);
  }
}
extern "C" void or_qkv_rope(float *q_out, uint16_t *k_cache, uint16_t *v_cache, const float *q, const float *k, const float *v,
                            const float *q_norm_w, const float *k_norm_w, uint32_t nq, uint32_t nkv, uint32_t D,
                            uint32_t rot_dim, int k_eq_v, float theta, float eps, uint32_t clock, uint32_t slot) {
  std::vector<float> inv_freq(rot_dim / 2);
  or_rope_inv_freq(inv_freq.data(), rot_dim, theta);
  qkv_rope_token(q_out, k_cache, v_cache, q, k, v, q_norm_w, k_norm_w, nq, nkv, D, rot_dim, k_eq_v, inv_freq.data(), eps,
                 clock, slot);
}

// ----------------------------------------------------------------------------
// attention -- shaders/decode_attn.wgsl:24-218 (scores * scale, max from -1e9,
// exp, 1/(sum+1e-9), weighted V).  Cache entries are f16.
static void attn_head(float *out, const float *qh, const uint16_t *kc, const uint16_t *vc, const uint32_t *slots, uint32_t b,
                      uint32_t e, size_t kv_dim, uint32_t kvh, uint32_t D, float scale, float *scores) {
  uint32_t S = e - b;
  for (uint32_t i = 0; i < S; i++) {
    const uint16_t *kr = kc + (size_t)slots[b + i] * kv_dim + (size_t)kvh * D;
    float dot = 0.0f;
    for (uint32_t d = 0; d < D; d++) dot += qh[d] * or_f16_to_f32(kr[d]);
    scores[i] = dot * scale;
  }
  float mx = -1e9f;
  for (uint32_t i = 0; i < S; i++)
    if (scores[i] > mx) mx = scores[i];
  float sum = 0.0f;
  for (uint32_t i = 0; i < S; i++) {
    scores[i] = expf(scores[i] - mx);
    sum += scores[i];
  }
  float inv = 1.0f / (sum + 1e-9f);
  for (uint32_t d = 0; d < D; d++) out[d] = 0.0f;
  for (uint32_t i = 0; i < S; i++) {
    float p = scores[i] * inv;
    const uint16_t *vr = vc + (size_t)slots[b + i] * kv_dim + (size_t)kvh * D;
    for (uint32_t d = 0; d < D; d++) out[d] += p * or_f16_to_f32(vr[d]);
  }
}
extern "C" void or_decode_attn(float *out, const float *q, const uint16_t *k_cache, const uint16_t *v_cache,
                               const uint32_t *slots, uint32_t S, uint32_t nq, uint32_t nkv, uint32_t D, float scale) {
  std::vector<float> scores(S + 1);
  uint32_t ratio = nq / nkv;
  for (uint32_t h = 0; h < nq; h++)
    attn_head(out + (size_t)h * D, q + (size_t)h * D, k_cache, v_cache, slots, 0, S, (size_t)nkv * D, h / ratio, D, scale,
              scores.data());
}

// ----------------------------------------------------------------------------
// sampling -- shaders/topk_pass1.wgsl:17-19 (softcap), kernels.zig:133-143 (argmax)
extern "C" float or_softcap(float v) { return 30.0f * tanhf(v * (1.0f / 30.0f)); }
extern "C" void or_topk64(uint32_t *ids, float *vals, const float *logits, size_t V) {
  std::vector<float> sc(V);
  std::vector<uint32_t> idx(V);
  for (size_t i = 0; i < V; i++) {
    sc[i] = or_softcap(logits[i]);
    idx[i] = (uint32_t)i;
  }
  size_t k = std::min<size_t>(64, V);
  std::partial_sort(idx.begin(), idx.begin() + k, idx.end(), [&](uint32_t a, uint32_t b) {
    if (sc[a] != sc[b]) return sc[a] > sc[b];
    return a < b;
  });
  for (size_t i = 0; i < 64; i++) {
    ids[i] = i < k ? idx[i] : 0;
    vals[i] = i < k ? sc[idx[i]] : -1e30f;
  }
}
extern "C" uint32_t or_argmax(const float *logits, size_t V) {
  uint32_t mi = 0;
  float mv = logits[0];
  for (size_t i = 1; i < V; i++)
    if (logits[i] > mv) {
      mv = logits[i];
      mi = (uint32_t)i;
    }
  return mi;
}
// src/sampler.zig:44-58 (isCritiqueToken) and :210-266 (sampleTopK, temp <= 0)
static bool is_critique(uint32_t t) {
  static const uint32_t c[] = {20470, 29202, 12429, 4491, 83675, 213110, 68755, 38403, 89429, 3643, 4573, 5503, 9675, 97485};
  for (uint32_t x : c)
    if (x == t) return true;
  return false;
}
extern "C" uint32_t or_sample_topk_greedy(const uint32_t *ids, const float *vals, size_t n, const uint32_t *recent,
                                          size_t n_recent, float rp, float fp, float pp, int sup_think, int sup_close,
                                          int sup_crit) {
  if (n == 0) return 0;
  bool has_pen = (rp > 1.0f || fp > 0.0f || pp > 0.0f);
  if ((!has_pen || recent == nullptr) && !sup_think && !sup_crit && !sup_close) return ids[0];
  static const uint32_t sup[] = {0, 258882, 258883, 255999, 256000, 256001, 255995, 255996, 255997, 255998};
  struct C {
    uint32_t id;
    float val;
  };
  std::vector<C> items;
  for (size_t i = 0; i < n; i++) {
    uint32_t id = ids[i];
    bool skip = false;
    for (uint32_t s : sup)
      if (id == s) skip = true;
    if (skip) continue;
    if (sup_think && id == 100) continue;
    if (sup_close && id == 101) continue;
    if (sup_crit && is_critique(id)) continue;
    items.push_back({id, vals[i]});
    if (items.size() == 64) break;
  }
  if (items.empty()) return ids[0];
  if (recent != nullptr && has_pen) {
    for (size_t i = 0; i < n_recent; i++) {
      uint32_t tok = recent[i];
      bool seen = false;
      for (size_t j = 0; j < i; j++)
        if (recent[j] == tok) seen = true;
      if (seen) continue;
      size_t count = 0;
      for (size_t j = 0; j < n_recent; j++)
        if (recent[j] == tok) count++;
      for (auto &it : items)
        if (it.id == tok) {
          if (rp > 1.0f) it.val = it.val > 0.0f ? it.val / rp : it.val * rp;
          it.val -= pp + ((float)count * fp);
        }
    }
    std::stable_sort(items.begin(), items.end(), [](const C &a, const C &b) { return a.val > b.val; });
  }
  return items[0].id;
}

// Zig's std.Random.DefaultPrng (Xoshiro256++ by Blackman & Vigna, 256-bit state filled
// by SplitMix64 from the seed: std/Random/Xoshiro256.zig init/seed/next) and
// Random.float(f32) (std/Random.zig: 23 random mantissa bits, the exponent from the
// leading zeros of the remaining bits of the same 64-bit draw).
static inline uint64_t or_rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }
extern "C" void or_prng_seed(uint64_t *st, uint64_t seed) {
  uint64_t z0 = seed;
  for (int i = 0; i < 4; i++) {  // SplitMix64.next
    z0 += 0x9e3779b97f4a7c15ull;
    uint64_t z = z0;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    st[i] = z ^ (z >> 31);
  }
}
extern "C" uint64_t or_prng_next(uint64_t *s) {
  const uint64_t r = or_rotl(s[0] + s[3], 23) + s[0];
  const uint64_t t = s[1] << 17;
  s[2] ^= s[0];
  s[3] ^= s[1];
  s[1] ^= s[2];
  s[0] ^= s[3];
  s[2] ^= t;
  s[3] = or_rotl(s[3], 45);
  return r;
}
extern "C" float or_prng_float(uint64_t *s) {
  const uint64_t rnd = or_prng_next(s);
  uint32_t lz = rnd ? (uint32_t)__builtin_clzll(rnd) : 64u;
  if (lz >= 41) {
    const uint64_t r2 = or_prng_next(s);
    lz = 41 + (r2 ? (uint32_t)__builtin_clzll(r2) : 64u);
    if (lz == 41 + 64) lz += (uint32_t)__builtin_clz((uint32_t)or_prng_next(s) | 0x7FFu);
  }
  const uint32_t bits = ((126u - lz) << 23) | ((uint32_t)rnd & 0x7FFFFFu);
  float f;
  memcpy(&f, &bits, 4);
  return f;
}
// Sampler.sampleTopK (src/sampler.zig:217-317): suppression, penalties with a stable
// re-sort, then temperature softmax, min-p, top-p and one draw.  params: temp, top_p,
// min_p, repeat, frequency, presence; flags: bit 0 suppress_thinking, bit 1
// suppress_critique, bit 2 suppress_channel_close.  recent NULL = no recent tokens.
extern "C" uint32_t or_sample_topk(const uint32_t *ids, const float *vals, size_t n, const uint32_t *recent,
                                   size_t n_recent, const float *params, int flags, uint64_t *prng) {
  const float temp = params[0], top_p = params[1], min_p = params[2], rp = params[3], fp = params[4], pp = params[5];
  const int sup_think = flags & 1, sup_crit = (flags >> 1) & 1, sup_close = (flags >> 2) & 1;
  if (n == 0) return 0;
  const bool has_pen = (rp > 1.0f || fp > 0.0f || pp > 0.0f);
  if (temp <= 0.0f && (!has_pen || recent == nullptr) && !sup_think && !sup_crit && !sup_close) return ids[0];
  static const uint32_t sup[] = {0, 258882, 258883, 255999, 256000, 256001, 255995, 255996, 255997, 255998};
  struct C {
    uint32_t id;
    float val;
  };
  std::vector<C> items;
  for (size_t i = 0; i < n; i++) {
    const uint32_t id = ids[i];
    bool skip = false;
    for (uint32_t x : sup)
      if (id == x) skip = true;
    if (skip || (sup_think && id == 100) || (sup_close && id == 101) || (sup_crit && is_critique(id))) continue;
    items.push_back({id, vals[i]});
    if (items.size() == 64) break;
  }
  if (items.empty()) return ids[0];
  if (recent != nullptr && has_pen) {
    for (size_t i = 0; i < n_recent; i++) {
      const uint32_t tok = recent[i];
      bool seen = false;
      for (size_t j = 0; j < i; j++)
        if (recent[j] == tok) seen = true;
      if (seen) continue;
      size_t count = 0;
      for (size_t j = 0; j < n_recent; j++)
        if (recent[j] == tok) count++;
      for (auto &it : items)
        if (it.id == tok) {
          if (rp > 1.0f) it.val = it.val > 0.0f ? it.val / rp : it.val * rp;
          it.val -= pp + ((float)count * fp);
        }
    }
    std::stable_sort(items.begin(), items.end(), [](const C &a, const C &b) { return a.val > b.val; });
  }
  if (temp <= 0.0f) return items[0].id;
  const size_t K = items.size();
  float probs[64];
  float max_scaled = -1e9f;
  for (size_t i = 0; i < K; i++) {
    probs[i] = items[i].val / temp;
    if (probs[i] > max_scaled) max_scaled = probs[i];
  }
  float sum = 0.0f;
  for (size_t i = 0; i < K; i++) {
    probs[i] = std::exp(probs[i] - max_scaled);
    sum += probs[i];
  }
  for (size_t i = 0; i < K; i++) probs[i] /= sum;
  const float p_thresh = probs[0] * min_p;
  size_t valid_k = 0;
  float valid_sum = 0.0f;
  for (size_t i = 0; i < K; i++) {
    if (probs[i] >= p_thresh) {
      valid_k = i + 1;
      valid_sum += probs[i];
    } else {
      break;
    }
  }
  if (valid_k == 0) valid_k = 1;
  for (size_t i = 0; i < valid_k; i++) probs[i] /= valid_sum;
  float cum_p = 0.0f;
  size_t cutoff = 0;
  for (size_t i = 0; i < valid_k; i++) {
    cum_p += probs[i];
    cutoff = i + 1;
    if (cum_p >= top_p) break;
  }
  const float r = or_prng_float(prng) * cum_p;
  float acc = 0.0f;
  uint32_t chosen = items[0].id;
  for (size_t i = 0; i < cutoff; i++) {
    acc += probs[i];
    if (acc >= r) {
      chosen = items[i].id;
      break;
    }
  }
  return chosen;
}

// ----------------------------------------------------------------------------
// batched prefill ops -- shaders/batch_gemm_q4.wgsl:26-160 (Y[t*M + r]),
// batch_fused_mlp_q4.wgsl:33-196, batch_rmsnorm.wgsl, batch_add_rmsnorm.wgsl,
// batch_qkv_rope.wgsl:29-176, batch_causal_attn.wgsl:25-223
// A row's nibbles decoded once to (q - 8) floats; the per-block arithmetic is the
// same sequence as q4_row_dot (four 8-term chains, then acc += s * dot).
static void decode_q4_row(const uint32_t *row, size_t nb, float *n, float *s) {
  for (size_t b = 0; b < nb; b++) {
    const uint32_t *blk = row + b * 5;
    s[b] = or_f16_to_f32((uint16_t)(blk[0] & 0xFFFFu));
    for (int w = 0; w < 4; w++)
      for (int k = 0; k < 8; k++) n[b * 32 + w * 8 + k] = (float)((blk[1 + w] >> (4 * k)) & 0xFu) - 8.0f;
  }
}
static inline float q4_dec_dot(const float *n, const float *s, const float *x, size_t nb) {
  float acc = 0.0f;
  for (size_t b = 0; b < nb; b++) {
    const float *nn = n + b * 32, *xb = x + b * 32;
    float u[4];
    for (int w = 0; w < 4; w++) {
      const float *a = nn + w * 8, *xa = xb + w * 8;
      u[w] = a[0] * xa[0] + a[1] * xa[1] + a[2] * xa[2] + a[3] * xa[3] + a[4] * xa[4] + a[5] * xa[5] + a[6] * xa[6] +
             a[7] * xa[7];
    }
    float dot = u[0] + u[1] + u[2] + u[3];
    acc += s[b] * dot;
  }
  return acc;
}
extern "C" void or_batch_gemm_q4(float *Y, const uint32_t *W, const float *X, size_t N, size_t M, size_t K, int threads) {
  size_t nb = K / 32;
  parallel_rows(M, threads, [&](size_t b, size_t e) {
    std::vector<float> n(K), s(nb);
    for (size_t r = b; r < e; r++) {
      decode_q4_row(W + r * nb * 5, nb, n.data(), s.data());
      for (size_t t = 0; t < N; t++) Y[t * M + r] = q4_dec_dot(n.data(), s.data(), X + t * K, nb);
    }
  });
}
extern "C" void or_batch_fused_mlp_q4(float *Y, const uint32_t *Wg, const uint32_t *Wu, const float *X, size_t N, size_t M,
                                      size_t K, int threads) {
  size_t nb = K / 32;
  parallel_rows(M, threads, [&](size_t b, size_t e) {
    std::vector<float> ng(K), sg(nb), nu(K), su(nb);
    for (size_t r = b; r < e; r++) {
      decode_q4_row(Wg + r * nb * 5, nb, ng.data(), sg.data());
      decode_q4_row(Wu + r * nb * 5, nb, nu.data(), su.data());
      for (size_t t = 0; t < N; t++) {
        float g = q4_dec_dot(ng.data(), sg.data(), X + t * K, nb);
        float u = q4_dec_dot(nu.data(), su.data(), X + t * K, nb);
        Y[t * M + r] = or_gelu_tanh(g) * u;
      }
    }
  });
}
extern "C" void or_batch_rmsnorm(float *Y, const float *X, const float *w, size_t N, size_t H, float eps) {
  for (size_t t = 0; t < N; t++) or_rmsnorm(Y + t * H, X + t * H, w, H, eps);
}
extern "C" void or_batch_add_rmsnorm(float *X, const float *R, const float *w, float *Y, size_t N, size_t H, float eps,
                                     float scalar) {
  for (size_t t = 0; t < N; t++) or_add_rmsnorm(X + t * H, R + t * H, w, Y + t * H, H, eps, scalar);
}
extern "C" void or_batch_qkv_rope(float *q_out, uint16_t *k_cache, uint16_t *v_cache, const float *q, const float *k,
                                  const float *v, const float *q_norm_w, const float *k_norm_w, uint32_t N, uint32_t nq,
                                  uint32_t nkv, uint32_t D, uint32_t rot_dim, int k_eq_v, float theta, float eps,
                                  uint32_t start_clock, const uint32_t *slots, uint32_t slot_offset) {
  std::vector<float> inv_freq(rot_dim / 2);
  or_rope_inv_freq(inv_freq.data(), rot_dim, theta);
  size_t qd = (size_t)nq * D, kvd = (size_t)nkv * D;
  for (uint32_t t = 0; t < N; t++)
    qkv_rope_token(q_out + t * qd, k_cache, v_cache, q + t * qd, k + t * kvd, v + t * kvd, q_norm_w, k_norm_w, nq, nkv, D,
                   rot_dim, k_eq_v, inv_freq.data(), eps, start_clock + t, slots[slot_offset + t]);
}
extern "C" void or_batch_causal_attn(float *out, const float *q, const uint16_t *k_cache, const uint16_t *v_cache,
                                     const uint32_t *slots, uint32_t N, uint32_t num_prev, uint32_t nq, uint32_t nkv,
                                     uint32_t D, float scale, int is_sliding, int threads) {
  uint32_t ratio = nq / nkv;
  size_t qd = (size_t)nq * D;
  parallel_rows(N, threads, [&](size_t b, size_t e) {
    std::vector<float> scores(num_prev + N + 1);
    for (size_t t = b; t < e; t++) {
      uint32_t S = num_prev + (uint32_t)t + 1;
      uint32_t start = (is_sliding && S > 1024) ? S - 1024 : 0;  // batch_causal_attn.wgsl:52-53
      for (uint32_t h = 0; h < nq; h++)
        attn_head(out + t * qd + (size_t)h * D, q + t * qd + (size_t)h * D, k_cache, v_cache, slots, start, S,
                  (size_t)nkv * D, h / ratio, D, scale, scores.data());
    }
  });
}

// ----------------------------------------------------------------------------
// ring buffer -- src/ring_buffer.zig (metadata; K/V live in the model)
namespace {
const size_t TOTAL_SLOTS = 4096, UPPER_RECALL = 128, MAX_BOUNDARIES = 1024;
}
struct or_ring {
  size_t num_layers, num_anchors, total_ingested;
  std::vector<size_t> clocks;
  std::vector<uint8_t> active;
  std::vector<float> mass;
  size_t boundaries[1024];
  int btypes[1024];
  float bsal[1024];
  size_t nb;
};
extern "C" or_ring *or_ring_create(uint32_t num_layers, uint32_t num_anchors) {
  or_ring *r = new or_ring();
  r->num_layers = num_layers;
  r->num_anchors = num_anchors;
  r->total_ingested = 0;
  r->clocks.assign((size_t)num_layers * TOTAL_SLOTS, 0);
  r->active.assign((size_t)num_layers * TOTAL_SLOTS, 0);
  r->mass.assign((size_t)num_layers * TOTAL_SLOTS, 0.0f);
  r->nb = 0;
  memset(r->boundaries, 0, sizeof(r->boundaries));
  return r;
}
extern "C" void or_ring_destroy(or_ring *r) { delete r; }
extern "C" void or_ring_reset(or_ring *r) {
  std::fill(r->clocks.begin(), r->clocks.end(), 0);
  std::fill(r->active.begin(), r->active.end(), 0);
  std::fill(r->mass.begin(), r->mass.end(), 0.0f);
  r->total_ingested = 0;
  r->nb = 0;
}
// ring_buffer.zig:101-103
extern "C" void or_ring_set_num_anchors(or_ring *r, size_t n) {
  r->num_anchors = std::min(n, TOTAL_SLOTS - UPPER_RECALL - 64);
}
extern "C" size_t or_ring_num_anchors(const or_ring *r) { return r->num_anchors; }
extern "C" size_t or_ring_total_ingested(const or_ring *r) { return r->total_ingested; }
static size_t recall_slots() { return TOTAL_SLOTS < UPPER_RECALL * 2 ? 0 : UPPER_RECALL; }  // :104-107
extern "C" size_t or_ring_recall_start(const or_ring *, size_t) { return TOTAL_SLOTS - recall_slots(); }
extern "C" size_t or_ring_window_size(const or_ring *r, size_t layer) {  // :111-114
  size_t start = or_ring_recall_start(r, layer);
  return start > r->num_anchors ? start - r->num_anchors : 1;
}
extern "C" size_t or_ring_get_slot_index(const or_ring *r, size_t layer, size_t clock) {  // :118-121
  if (clock < r->num_anchors) return clock;
  return r->num_anchors + ((clock - r->num_anchors) % or_ring_window_size(r, layer));
}
extern "C" size_t or_ring_activate_slot(or_ring *r, size_t layer, size_t clock) {  // :123-131
  size_t slot = or_ring_get_slot_index(r, layer, clock);
  size_t i = layer * TOTAL_SLOTS + slot;
  r->clocks[i] = clock;
  r->active[i] = 1;
  r->mass[i] = 0.0f;
  if (layer == 0 && clock >= r->total_ingested) r->total_ingested = clock + 1;
  return slot;
}
extern "C" void or_ring_deactivate_slot(or_ring *r, size_t layer, size_t clock) {  // :133-141
  size_t slot = or_ring_get_slot_index(r, layer, clock);
  size_t i = layer * TOTAL_SLOTS + slot;
  if (r->clocks[i] == clock) {
    r->active[i] = 0;
    r->clocks[i] = 0;
    r->mass[i] = 0.0f;
  }
}
extern "C" void or_ring_rollback_clock(or_ring *r, size_t target) {  // :143-151
  if (target >= r->total_ingested) return;
  for (size_t c = target; c < r->total_ingested; c++)
    for (size_t l = 0; l < r->num_layers; l++) or_ring_deactivate_slot(r, l, c);
  r->total_ingested = target;
}
extern "C" void or_ring_write_kv_meta(or_ring *r, size_t layer, size_t clock) {  // :254-264 (metadata part)
  size_t slot = or_ring_get_slot_index(r, layer, clock);
  size_t i = layer * TOTAL_SLOTS + slot;
  r->clocks[i] = clock;
  r->active[i] = 1;
  if (layer == 0 && clock >= r->total_ingested) r->total_ingested = clock + 1;
}
extern "C" void or_ring_write_recall_meta(or_ring *r, size_t layer, size_t rank, size_t clock) {  // :273-281
  size_t slot = or_ring_recall_start(r, layer) + rank;
  if (slot >= TOTAL_SLOTS) return;
  size_t i = layer * TOTAL_SLOTS + slot;
  r->clocks[i] = clock;
  r->active[i] = 1;
}
extern "C" void or_ring_clear_recall(or_ring *r) {  // :266-271
  for (size_t l = 0; l < r->num_layers; l++) {
    size_t base = l * TOTAL_SLOTS + or_ring_recall_start(r, l);
    for (size_t s = 0; s < recall_slots(); s++) r->active[base + s] = 0;
  }
}
extern "C" void or_ring_mark_boundary(or_ring *r, size_t clock, int span_type, float salience) {  // :79-90
  if (r->nb > 0 && r->boundaries[(r->nb - 1) % MAX_BOUNDARIES] == clock) {
    r->btypes[(r->nb - 1) % MAX_BOUNDARIES] = span_type;
    r->bsal[(r->nb - 1) % MAX_BOUNDARIES] = salience;
    return;
  }
  size_t i = r->nb % MAX_BOUNDARIES;
  r->boundaries[i] = clock;
  r->btypes[i] = span_type;
  r->bsal[i] = salience;
  r->nb++;
}
static size_t snap_to_boundary(const or_ring *r, size_t raw) {  // :92-100
  if (raw <= r->num_anchors || r->nb == 0) return raw;
  size_t start = r->nb > MAX_BOUNDARIES ? r->nb - MAX_BOUNDARIES : 0;
  for (size_t i = start; i < r->nb; i++) {
    size_t b = r->boundaries[i % MAX_BOUNDARIES];
    if (b >= raw) return b;
  }
  return raw;
}
extern "C" void or_ring_record_attention(or_ring *r, size_t layer, size_t slot, float m) {  // :153-157
  if (layer < r->num_layers && slot < TOTAL_SLOTS) r->mass[layer * TOTAL_SLOTS + slot] += m;
}
extern "C" float or_ring_attention_mass(const or_ring *r, size_t layer, size_t slot) {
  return (layer < r->num_layers && slot < TOTAL_SLOTS) ? r->mass[layer * TOTAL_SLOTS + slot] : 0.0f;
}
extern "C" float or_ring_slot_salience(const or_ring *r, size_t slot) {  // :163-168
  if (slot >= TOTAL_SLOTS) return 0.0f;
  float sum = 0.0f;
  for (size_t l = 0; l < r->num_layers; l++) sum += r->mass[l * TOTAL_SLOTS + slot];
  return sum / (float)r->num_layers;
}
extern "C" float or_ring_working_set_gini(const or_ring *r) {  // :170-197
  std::vector<float> s;
  float total = 0.0f;
  size_t w_end = or_ring_recall_start(r, 0);
  for (size_t slot = r->num_anchors; slot < w_end; slot++)
    if (r->active[slot]) {
      float v = or_ring_slot_salience(r, slot);
      s.push_back(v);
      total += v;
    }
  if (s.size() < 2 || total <= 0.0f) return 1.0f;
  std::sort(s.begin(), s.end());
  float ws = 0.0f;
  for (size_t i = 0; i < s.size(); i++) ws += (float)(i + 1) * s[i];
  float n = (float)s.size();
  float g = (2.0f * ws) / (n * total) - (n + 1.0f) / n;
  return std::max(0.0f, std::min(1.0f, g));
}
extern "C" int or_ring_is_saturated(const or_ring *r, float cap, float gini_t) {  // :199-213
  size_t w_end = or_ring_recall_start(r, 0);
  size_t tier2 = w_end > r->num_anchors ? w_end - r->num_anchors : 1;
  size_t cnt = 0;
  for (size_t slot = r->num_anchors; slot < w_end; slot++)
    if (r->active[slot]) cnt++;
  float fill = (float)cnt / (float)tier2;
  if (fill < cap) return 0;
  return or_ring_working_set_gini(r) < gini_t;
}
extern "C" size_t or_ring_evict_low_salience(or_ring *r, size_t min_clock, size_t max_clock, size_t evict_count) {
  // :215-252
  if (min_clock >= max_clock || evict_count == 0) return 0;
  struct Cand {
    size_t slot;
    float sal;
  };
  std::vector<Cand> c;
  for (size_t clk = min_clock; clk < max_clock + 1; clk++) {
    if (clk < r->num_anchors) continue;
    size_t slot = or_ring_get_slot_index(r, 0, clk);
    if (r->active[slot] && r->clocks[slot] == clk && c.size() < 1024) c.push_back({slot, or_ring_slot_salience(r, slot)});
  }
  if (c.empty()) return 0;
  std::stable_sort(c.begin(), c.end(), [](const Cand &a, const Cand &b) { return a.sal < b.sal; });
  size_t n = std::min(evict_count, c.size());
  for (size_t i = 0; i < n; i++)
    for (size_t l = 0; l < r->num_layers; l++) r->active[l * TOTAL_SLOTS + c[i].slot] = 0;
  return n;
}
extern "C" int or_ring_is_active(const or_ring *r, size_t layer, size_t slot) { return r->active[layer * TOTAL_SLOTS + slot]; }
extern "C" size_t or_ring_slot_clock(const or_ring *r, size_t layer, size_t slot) { return r->clocks[layer * TOTAL_SLOTS + slot]; }
extern "C" size_t or_ring_active_slots(const or_ring *r, size_t layer, size_t clock, int is_sliding, size_t sliding_window,
                                       uint32_t *out) {  // :287-333
  size_t off = layer * TOTAL_SLOTS, count = 0;
  size_t eff = is_sliding ? sliding_window : or_ring_window_size(r, layer);
  size_t raw_min = clock >= eff ? clock - eff + 1 : 0;
  size_t min_valid = is_sliding ? raw_min : snap_to_boundary(r, raw_min);
  size_t anchor_limit = std::min(clock + 1, r->num_anchors);
  for (size_t s = 0; s < anchor_limit; s++)
    if (r->active[off + s] && (!is_sliding || s >= min_valid)) out[count++] = (uint32_t)s;
  size_t dyn = std::max(min_valid, r->num_anchors);
  if (clock >= dyn)
    for (size_t c = dyn; c < clock + 1; c++) {
      size_t slot = or_ring_get_slot_index(r, layer, c);
      if (r->active[off + slot] && r->clocks[off + slot] == c) out[count++] = (uint32_t)slot;
    }
  if (!is_sliding)
    for (size_t s = or_ring_recall_start(r, layer); s < TOTAL_SLOTS; s++) {
      if (!r->active[off + s]) continue;
      if (r->clocks[off + s] <= clock) out[count++] = (uint32_t)s;
    }
  return count;
}
extern "C" size_t or_ring_prefill_prev_slots(const or_ring *r, size_t layer, size_t start_clock, size_t chunk_len,
                                             uint32_t *out) {  // :335-380
  size_t off = layer * TOTAL_SLOTS, count = 0;
  if (start_clock == 0 || chunk_len == 0) return 0;
  size_t end_clock = start_clock + chunk_len - 1;
  size_t w = or_ring_window_size(r, layer);
  size_t raw_min = end_clock >= w ? end_clock - w + 1 : 0;
  size_t min_valid = snap_to_boundary(r, raw_min);
  size_t anchor_limit = std::min(start_clock, r->num_anchors);
  for (size_t s = 0; s < anchor_limit; s++)
    if (r->active[off + s]) out[count++] = (uint32_t)s;
  size_t dyn = std::max(min_valid, r->num_anchors);
  if (start_clock > dyn)
    for (size_t c = dyn; c < start_clock; c++) {
      size_t slot = or_ring_get_slot_index(r, layer, c);
      if (r->active[off + slot] && r->clocks[off + slot] == c) out[count++] = (uint32_t)slot;
    }
  for (size_t s = or_ring_recall_start(r, layer); s < TOTAL_SLOTS; s++) {
    if (!r->active[off + s]) continue;
    if (r->clocks[off + s] < start_clock) out[count++] = (uint32_t)s;
  }
  return count;
}

// ----------------------------------------------------------------------------
// whole model -- GPU dispatch order (src/gpu/model_dispatch.zig:10-45 decode;
// src/gpu/batch_dispatch.zig:55-151 prefill).  Layer-0 input norm is explicit,
// every later input norm is fused into the previous layer's post-FFN add
// (model_gpu.zig:160-163); the LM head is the Q8_0 table (model_gpu.zig:157).
struct or_model {
  or_model_cfg cfg;
  std::vector<or_layer> layers;
  const uint32_t *lm_head;
  const float *final_norm;
  int threads;
  std::vector<std::vector<uint16_t>> kc, vc;
  std::vector<float> x, normed, q, k, v, qo, attn, mlp, act, logits;
  std::vector<float> inv_freq_s, inv_freq_f;
};
extern "C" or_model *or_model_create(const or_model_cfg *cfg, const or_layer *layers, const uint32_t *lm_head_q8,
                                     const float *final_norm, int threads) {
  or_model *m = new or_model();
  m->cfg = *cfg;
  m->layers.assign(layers, layers + cfg->layers);
  m->lm_head = lm_head_q8;
  m->final_norm = final_norm;
  m->threads = threads;
  size_t kvd = (size_t)cfg->n_kv * cfg->head_dim;
  m->kc.assign(cfg->layers, std::vector<uint16_t>(TOTAL_SLOTS * kvd, 0));
  m->vc.assign(cfg->layers, std::vector<uint16_t>(TOTAL_SLOTS * kvd, 0));
  m->inv_freq_s.resize(cfg->rot_dim / 2);
  m->inv_freq_f.resize(cfg->rot_dim / 2);
  or_rope_inv_freq(m->inv_freq_s.data(), cfg->rot_dim, cfg->theta_sliding);
  or_rope_inv_freq(m->inv_freq_f.data(), cfg->rot_dim, cfg->theta_full);
  return m;
}
extern "C" void or_model_destroy(or_model *m) { delete m; }
extern "C" void or_model_reset_kv(or_model *m) {
  for (auto &c : m->kc) std::fill(c.begin(), c.end(), 0);
  for (auto &c : m->vc) std::fill(c.begin(), c.end(), 0);
}
extern "C" const float *or_model_x(const or_model *m) { return m->x.data(); }
extern "C" const float *or_model_normed_x(const or_model *m) { return m->normed.data(); }
extern "C" const uint16_t *or_model_k_cache(const or_model *m, uint32_t l) { return m->kc[l].data(); }
extern "C" const uint16_t *or_model_v_cache(const or_model *m, uint32_t l) { return m->vc[l].data(); }

static void logits_topk(or_model *m, const float *normed, uint32_t *ids, float *vals) {
  const or_model_cfg &c = m->cfg;
  m->logits.resize(c.vocab);
  or_gemv_q8(m->logits.data(), m->lm_head, normed, c.vocab, c.hidden, m->threads);
  or_topk64(ids, vals, m->logits.data(), c.vocab);
}

extern "C" uint32_t or_model_forward_token(or_model *m, const float *x_in, uint32_t clock, uint32_t slot,
                                           const uint32_t *active, uint32_t n_active, const uint32_t *sliding,
                                           uint32_t n_sliding, uint32_t *topk_ids, float *topk_vals) {
  const or_model_cfg &c = m->cfg;
  size_t H = c.hidden, I = c.inter, D = c.head_dim, qd = (size_t)c.n_q * D, kvd = (size_t)c.n_kv * D;
  int T = m->threads;
  m->x.assign(x_in, x_in + H);
  m->normed.resize(H);
  m->q.resize(qd);
  m->k.resize(kvd);
  m->v.resize(kvd);
  m->qo.resize(qd);
  m->attn.resize(qd);
  m->mlp.resize(H);
  m->act.resize(I);
  for (uint32_t li = 0; li < c.layers; li++) {
    const or_layer &L = m->layers[li];
    bool full = c.layer_full[li] != 0;
    if (li == 0) or_rmsnorm(m->normed.data(), m->x.data(), L.input_norm, H, c.eps);
    or_gemv_q4(m->q.data(), L.wq, m->normed.data(), qd, H, T);
    or_gemv_q4(m->k.data(), L.wk, m->normed.data(), kvd, H, T);
    or_gemv_q4(m->v.data(), L.wv, m->normed.data(), kvd, H, T);
    qkv_rope_token(m->qo.data(), m->kc[li].data(), m->vc[li].data(), m->q.data(), m->k.data(), m->v.data(), L.q_norm,
                   L.k_norm, c.n_q, c.n_kv, (uint32_t)D, c.rot_dim, 0, full ? m->inv_freq_f.data() : m->inv_freq_s.data(),
                   c.eps, clock, slot);
    // decode uses layer 0's lists for every layer (model_dispatch.zig:133-135, forward.zig:44-47)
    const uint32_t *sl = full ? active : sliding;
    uint32_t S = full ? n_active : n_sliding;
    or_decode_attn(m->attn.data(), m->qo.data(), m->kc[li].data(), m->vc[li].data(), sl, S, c.n_q, c.n_kv, (uint32_t)D, 1.0f);
    or_gemv_q4(m->mlp.data(), L.wo, m->attn.data(), H, qd, T);
    if (L.post_attn_norm) or_rmsnorm(m->mlp.data(), m->mlp.data(), L.post_attn_norm, H, c.eps);
    or_add_rmsnorm(m->x.data(), m->mlp.data(), L.pre_ffn_norm, m->normed.data(), H, c.eps, 1.0f);
    or_fused_mlp_q4(m->act.data(), L.wg, L.wu, m->normed.data(), I, H, T);
    or_gemv_q4(m->mlp.data(), L.wd, m->act.data(), H, I, T);
    if (L.post_ffn_norm) or_rmsnorm(m->mlp.data(), m->mlp.data(), L.post_ffn_norm, H, c.eps);
    const float *next = (li + 1 < c.layers) ? m->layers[li + 1].input_norm : m->final_norm;
    or_add_rmsnorm(m->x.data(), m->mlp.data(), next, m->normed.data(), H, c.eps, L.layer_scalar);
  }
  uint32_t ids[64];
  float vals[64];
  logits_topk(m, m->normed.data(), ids, vals);
  if (topk_ids) memcpy(topk_ids, ids, sizeof(ids));
  if (topk_vals) memcpy(topk_vals, vals, sizeof(vals));
  return ids[0];
}

extern "C" uint32_t or_model_prefill(or_model *m, const float *X_in, uint32_t N, const uint32_t *slots, uint32_t start_clock,
                                     uint32_t n_prev, uint32_t *topk_ids, float *topk_vals) {
  const or_model_cfg &c = m->cfg;
  size_t H = c.hidden, I = c.inter, D = c.head_dim, qd = (size_t)c.n_q * D, kvd = (size_t)c.n_kv * D;
  int T = m->threads;
  std::vector<float> X(X_in, X_in + (size_t)N * H), NX((size_t)N * H), Q(N * qd), K(N * kvd), Vv(N * kvd), QO(N * qd),
      A(N * qd), MO((size_t)N * H), ACT((size_t)N * I);
  for (uint32_t li = 0; li < c.layers; li++) {
    const or_layer &L = m->layers[li];
    bool full = c.layer_full[li] != 0;
    if (li == 0) or_batch_rmsnorm(NX.data(), X.data(), L.input_norm, N, H, c.eps);
    or_batch_gemm_q4(Q.data(), L.wq, NX.data(), N, qd, H, T);
    or_batch_gemm_q4(K.data(), L.wk, NX.data(), N, kvd, H, T);
    or_batch_gemm_q4(Vv.data(), L.wv, NX.data(), N, kvd, H, T);
    or_batch_qkv_rope(QO.data(), m->kc[li].data(), m->vc[li].data(), Q.data(), K.data(), Vv.data(), L.q_norm, L.k_norm, N,
                      c.n_q, c.n_kv, (uint32_t)D, c.rot_dim, 0, full ? c.theta_full : c.theta_sliding, c.eps, start_clock,
                      slots, n_prev);
    or_batch_causal_attn(A.data(), QO.data(), m->kc[li].data(), m->vc[li].data(), slots, N, n_prev, c.n_q, c.n_kv,
                         (uint32_t)D, 1.0f, full ? 0 : 1, T);
    or_batch_gemm_q4(MO.data(), L.wo, A.data(), N, H, qd, T);
    if (L.post_attn_norm) or_batch_rmsnorm(MO.data(), MO.data(), L.post_attn_norm, N, H, c.eps);
    or_batch_add_rmsnorm(X.data(), MO.data(), L.pre_ffn_norm, NX.data(), N, H, c.eps, 1.0f);
    or_batch_fused_mlp_q4(ACT.data(), L.wg, L.wu, NX.data(), N, I, H, T);
    or_batch_gemm_q4(MO.data(), L.wd, ACT.data(), N, H, I, T);
    if (L.post_ffn_norm) or_batch_rmsnorm(MO.data(), MO.data(), L.post_ffn_norm, N, H, c.eps);
    const float *next = (li + 1 < c.layers) ? m->layers[li + 1].input_norm : m->final_norm;
    or_batch_add_rmsnorm(X.data(), MO.data(), next, NX.data(), N, H, c.eps, L.layer_scalar);
  }
  m->x.assign(X.begin() + (size_t)(N - 1) * H, X.begin() + (size_t)N * H);
  m->normed.assign(NX.begin() + (size_t)(N - 1) * H, NX.begin() + (size_t)N * H);
  uint32_t ids[64];
  float vals[64];
  logits_topk(m, m->normed.data(), ids, vals);
  if (topk_ids) memcpy(topk_ids, ids, sizeof(ids));
  if (topk_vals) memcpy(topk_vals, vals, sizeof(vals));
  return ids[0];
}

extern "C" void or_embed(float *x, const uint16_t *embed, const uint32_t *tokens, size_t n, size_t H) {
  float scale = sqrtf((float)H);  // forward.zig:33
  for (size_t t = 0; t < n; t++)
    for (size_t i = 0; i < H; i++) x[t * H + i] = or_bf16_to_f32(embed[(size_t)tokens[t] * H + i]) * scale;
}
