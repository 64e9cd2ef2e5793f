// sampler.cu -- Sampler.sampleTopK (src/sampler.zig:217-317) on the device.
//
// The reference samples on the host from the 64 candidates the GPU's top-k pass
// leaves (server/decode.zig:23-25): suppressed ids are dropped, the repeat /
// frequency / presence penalties of the recent tokens are applied and the
// candidates re-sorted (stable), then temperature softmax, min-p, top-p and one
// draw from the remaining mass.  Here one CTA does the same after the decode step,
// so a device-resident loop can sample without a host round trip per token:
//   * occurrence counts of the 64 candidate ids in the recent-token list are
//     counted by all threads (the list grows to thousands of tokens);
//   * the order-dependent rest -- stable insertion sort, the f32 sums of the
//     softmax, min-p and top-p in index order, the draw -- runs on one thread,
//     in the reference's operation order, so the choice is the reference's.
// The generator is Zig's std.Random.DefaultPrng (Xoshiro256++, seeded by
// SplitMix64) with Random.float(f32) (Zig 0.14 std/Random.zig), state in device
// memory, one 64-bit draw per sample.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.cuh"

namespace ch {

namespace {
constexpr int kSmThreads = 256;

CH_DEV uint64_t rotl64(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }
// Xoshiro256++ next() (Blackman & Vigna, the generator of Zig's DefaultPrng)
CH_DEV uint64_t xoshiro_next(uint64_t *s) {
  const uint64_t r = rotl64(s[0] + s[3], 23) + s[0];
  const uint64_t t = s[1] << 17;
  s[2] ^= s[0];
  s[3] ^= s[1];
  s[1] ^= s[2];
  s[0] ^= s[3];
  s[2] ^= t;
  s[3] = rotl64(s[3], 45);
  return r;
}
// Random.float(f32): 23 random mantissa bits, exponent from the leading zeros of the
// rest (every float in [0, 1) reachable, more draws only when 41 bits are zero)
CH_DEV float zig_float32(uint64_t *s) {
  const uint64_t rnd = xoshiro_next(s);
  uint32_t lz = (uint32_t)__clzll((long long)rnd);
  if (lz >= 41) {
    lz = 41 + (uint32_t)__clzll((long long)xoshiro_next(s));
    if (lz == 41 + 64) lz += (uint32_t)__clz((int)((uint32_t)xoshiro_next(s) | 0x7FFu));
  }
  const uint32_t mant = (uint32_t)rnd & 0x7FFFFFu;
  return __uint_as_float(((126u - lz) << 23) | mant);
}

// ids the reference never samples (sampler.zig:224) and the optional suppressions
CH_DEV bool suppressed(uint32_t id, const SamplerParams &p) {
  switch (id) {
    case 0: case 258882: case 258883: case 255999: case 256000: case 256001: case 255995: case 255996:
    case 255997: case 255998:
      return true;
    default:
      break;
  }
  if (p.suppress_thinking && id == 100) return true;
  if (p.suppress_channel_close && id == 101) return true;
  if (p.suppress_critique) {  // isCritiqueToken (sampler.zig:43-55)
    switch (id) {
      case 20470: case 29202: case 12429: case 4491: case 83675: case 213110: case 68755: case 38403: case 89429:
      case 3643: case 4573: case 5503: case 9675: case 97485:
        return true;
      default:
        break;
    }
  }
  return false;
}

__global__ void __launch_bounds__(kSmThreads) sample_topk_kernel(const SampleArgs a) {
  __shared__ uint32_t s_id[64], s_cnt[64];
  __shared__ float s_val[64], s_prob[64];
  __shared__ uint32_t s_k;
  const SamplerParams &p = a.p;
  const uint32_t n = min(a.n, 64u);
  const uint32_t n_recent = a.n_recent_dev ? min(*a.n_recent_dev, a.recent_cap) : a.n_recent;
  const bool has_pen = p.repeat_penalty > 1.0f || p.frequency_penalty > 0.0f || p.presence_penalty > 0.0f;
  const bool use_recent = a.recent != nullptr;
  // 1. candidates without the suppressed ids, in order (sampler.zig:221-231)
  if (threadIdx.x == 0) {
    uint32_t k = 0;
    for (uint32_t i = 0; i < n; i++)
      if (!suppressed(a.ids[i], p)) {
        s_id[k] = a.ids[i];
        s_val[k] = a.vals[i];
        k++;
      }
    s_k = k;
  }
  if (threadIdx.x < 64) s_cnt[threadIdx.x] = 0;
  __syncthreads();
  const uint32_t K = s_k;
  // 2. occurrences of each candidate id in the recent tokens
  if (use_recent && has_pen && K > 0) {
    const uint32_t item = threadIdx.x & 63u, part = threadIdx.x >> 6, parts = kSmThreads / 64;
    if (item < K) {
      const uint32_t id = s_id[item];
      uint32_t c = 0;
      for (uint32_t j = part; j < n_recent; j += parts) c += a.recent[j] == id ? 1u : 0u;
      if (c) atomicAdd(&s_cnt[item], c);
    }
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  uint32_t chosen;
  const bool greedy_early = p.temp <= 0.0f && (!has_pen || !use_recent) && !p.suppress_thinking &&
                            !p.suppress_critique && !p.suppress_channel_close;
  if (n == 0) {
    chosen = 0;
  } else if (greedy_early || K == 0) {  // sampler.zig:219-220,232
    chosen = a.ids[0];
  } else {
    if (use_recent && has_pen) {  // penalties (sampler.zig:234-259), then a stable descending re-sort
      for (uint32_t i = 0; i < K; i++) {
        if (!s_cnt[i]) continue;
        float v = s_val[i];
        if (p.repeat_penalty > 1.0f) v = v > 0.0f ? __fdiv_rn(v, p.repeat_penalty) : __fmul_rn(v, p.repeat_penalty);
        v = __fsub_rn(v, __fadd_rn(p.presence_penalty, __fmul_rn((float)s_cnt[i], p.frequency_penalty)));
        s_val[i] = v;
      }
      for (uint32_t i = 1; i < K; i++) {  // insertion sort: stable, like std.mem.sort
        const float v = s_val[i];
        const uint32_t id = s_id[i];
        uint32_t j = i;
        while (j > 0 && s_val[j - 1] < v) {
          s_val[j] = s_val[j - 1];
          s_id[j] = s_id[j - 1];
          j--;
        }
        s_val[j] = v;
        s_id[j] = id;
      }
    }
    if (p.temp <= 0.0f) {
      chosen = s_id[0];
    } else {
      // temperature softmax (sampler.zig:269-284)
      float mx = -1e9f;
      for (uint32_t i = 0; i < K; i++) {
        s_prob[i] = __fdiv_rn(s_val[i], p.temp);
        mx = s_prob[i] > mx ? s_prob[i] : mx;
      }
      float sum = 0.0f;
      for (uint32_t i = 0; i < K; i++) {
        s_prob[i] = expf(__fsub_rn(s_prob[i], mx));
        sum = __fadd_rn(sum, s_prob[i]);
      }
      for (uint32_t i = 0; i < K; i++) s_prob[i] = __fdiv_rn(s_prob[i], sum);
      // min-p (sampler.zig:286-297)
      const float thresh = __fmul_rn(s_prob[0], p.min_p);
      uint32_t valid_k = 0;
      float valid_sum = 0.0f;
      for (uint32_t i = 0; i < K; i++) {
        if (s_prob[i] >= thresh) {
          valid_k = i + 1;
          valid_sum = __fadd_rn(valid_sum, s_prob[i]);
        } else {
          break;
        }
      }
      if (valid_k == 0) valid_k = 1;
      for (uint32_t i = 0; i < valid_k; i++) s_prob[i] = __fdiv_rn(s_prob[i], valid_sum);
      // top-p (sampler.zig:299-305)
      float cum = 0.0f;
      uint32_t cutoff = 0;
      for (uint32_t i = 0; i < valid_k; i++) {
        cum = __fadd_rn(cum, s_prob[i]);
        cutoff = i + 1;
        if (cum >= p.top_p) break;
      }
      // the draw (sampler.zig:307-316)
      uint64_t st[4] = {a.prng[0], a.prng[1], a.prng[2], a.prng[3]};
      const float r = __fmul_rn(zig_float32(st), cum);
      a.prng[0] = st[0], a.prng[1] = st[1], a.prng[2] = st[2], a.prng[3] = st[3];
      float acc = 0.0f;
      chosen = s_id[0];
      for (uint32_t i = 0; i < cutoff; i++) {
        acc = __fadd_rn(acc, s_prob[i]);
        if (acc >= r) {
          chosen = s_id[i];
          break;
        }
      }
    }
  }
  *a.token_out = chosen;
  if (a.sp && a.token_hist && a.sp->step < a.hist_cap) a.token_hist[a.sp->step] = chosen;
  if (a.n_recent_dev && a.recent_w) {  // device loop: the sampled token joins the recent list
    const uint32_t c = *a.n_recent_dev;
    if (c < a.recent_cap) {
      a.recent_w[c] = chosen;
      *a.n_recent_dev = c + 1;
    }
  }
}
}  // namespace

cudaError_t launch_sample_topk(const SampleArgs &a, cudaStream_t s) {
  sample_topk_kernel<<<1, kSmThreads, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace ch
