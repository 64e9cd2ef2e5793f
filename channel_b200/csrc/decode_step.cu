// decode_step.cu -- one greedy decode token as ONE persistent kernel.
//
// Replaces the reference's per-token command buffer of ~12 dispatches per layer
// (src/gpu/model_dispatch.zig:226-342: fused_qkv_q4, qkv_rope, decode_attn,
// gemv_q4(O), rmsnorm/add_rmsnorm, fused_mlp_q4, gemv_q4(down), ..., gemv_q8 +
// topk_pass1/2) with a phase list executed by a cooperative grid of one CTA per
// SM:
//
//   per layer:  GEMV q|k|v  ->  ATTN  ->  GEMV o  ->  GEMV gate|up  ->  GEMV down
//   tail:       GEMV Q8 LM head  ->  TOPK
//
// B200 design.  A decode token is an HBM weight stream (7.2 GB for the 12B
// shape) with tiny activations in between.  Every warp owns a balanced share of
// the tiles of every GEMV phase and streams its shares of ALL phases back to
// back through its own bulk-copy (cp.async.bulk) stages, so the weight stream
// never drains at phase boundaries: weights do not depend on activations.  Only
// the compute waits, on a grid-wide barrier per phase.  GEMV outputs are left as
// per-warp partial row sums (no atomics, no fences in the GEMV) and the consumer
// phase sums them in a fixed order while building its input (norms, GELU*up,
// attention heads) -- deterministic, and the reduction rides on the L2 reads
// the consumer needs anyway.
#include <algorithm>

#include "common.cuh"
#include "core.cuh"
#include "decode_step.cuh"

namespace ch {

namespace {
constexpr int MK_NW = 16;  // warps per CTA (all stream + compute)
constexpr int MK_SPW = 2;  // bulk-copy stages per warp
constexpr int MK_CT = 6;   // tiles per stage
constexpr int MK_STAGE = MK_CT * kTileBytes;
constexpr int MK_THREADS = MK_NW * 32;
constexpr uint32_t kMinChunk = 64;
constexpr uint32_t kVecRows = 4096;  // rows staged per gather in the GEMV prologues
}  // namespace

int mk_warps() { return MK_NW; }

// ---------------------------------------------------------------------------
// balanced partition of T tiles over GW warps: warp w owns [w*q + min(w,rem), ...)
CH_DEV uint32_t part_begin(uint32_t w, uint32_t q, uint32_t rem) { return w * q + min(w, rem); }
CH_DEV uint32_t part_warp_of(uint32_t t, uint32_t q, uint32_t rem) {
  const uint32_t big = rem * (q + 1);
  return t < big ? t / (q + 1) : rem + (t - big) / q;
}

// CTA-level view of the same partition: CTA c owns tiles [cta_begin(c), cta_begin(c+1))
CH_DEV uint32_t cta_begin(const GemvOut &o, uint32_t c) { return part_begin(c * MK_NW, o.q, o.rem); }
CH_DEV uint32_t cta_of(const GemvOut &o, uint32_t t) { return part_warp_of(t, o.q, o.rem) / MK_NW; }

// Finished rows [r0, r1) of a GEMV output (act mode: finished acts) into shared
// memory: every row is final in `direct` after the phase barrier.
CH_DEV void gather_rows(const GemvOut &o, uint32_t r0, uint32_t r1, float *dst) {
  const uint32_t n = r1 - r0;
  for (uint32_t i = threadIdx.x * 4; i < n; i += blockDim.x * 4) {
    if (i + 4 <= n && ((r0 + i) & 3) == 0) {
      *reinterpret_cast<float4 *>(dst + i) = __ldcg(reinterpret_cast<const float4 *>(o.direct + r0 + i));
    } else {
      for (uint32_t e = i; e < min(n, i + 4); e++) dst[e] = __ldcg(&o.direct[r0 + e]);
    }
  }
  __syncthreads();
}

// grid barrier on a monotonically increasing arrival counter (bounded wait)
CH_DEV void grid_barrier(unsigned long long *arrive, unsigned long long target, uint32_t *err) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(arrive, 1ull);
    unsigned long long v;
    asm volatile("ld.acquire.gpu.u64 %0, [%1];" : "=l"(v) : "l"(arrive) : "memory");
    if (v < target) {
      const uint64_t t0 = globaltimer_ns();
      for (;;) {
        asm volatile("ld.acquire.gpu.u64 %0, [%1];" : "=l"(v) : "l"(arrive) : "memory");
        if (v >= target) break;
        if (globaltimer_ns() - t0 > 2000000000ull) {
          atomicOr(err, DEV_ERR_PEER_TIMEOUT);
          break;
        }
      }
    }
    __threadfence();
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// per-warp weight stream over the GEMV phases
struct Stream {
  uint32_t ph, ck;  // next chunk to issue: phase index, chunk index within the warp's share
};

CH_DEV uint32_t warp_chunks(const Phase &p, uint32_t gw) {
  const uint32_t tb = part_begin(gw, p.q, p.rem), te = part_begin(gw + 1, p.q, p.rem);
  return (te - tb + MK_CT - 1) / MK_CT;
}

// advance `s` to the next (phase, chunk) to issue; false when the step's stream is done
CH_DEV bool stream_next(const MegaArgs &a, uint32_t gw, Stream &s) {
  while (s.ph < a.nphases) {
    const Phase &p = a.phases[s.ph];
    if (p.kind == PH_GEMV && s.ck < warp_chunks(p, gw)) return true;
    s.ph++;
    s.ck = 0;
  }
  return false;
}

CH_DEV void stream_issue(const MegaArgs &a, uint32_t gw, Stream &s, uint8_t *stage, uint64_t *bar) {
  const Phase &p = a.phases[s.ph];
  const uint32_t tb = part_begin(gw, p.q, p.rem), te = part_begin(gw + 1, p.q, p.rem);
  const uint32_t t0 = tb + s.ck * MK_CT;
  const uint32_t bytes = min((uint32_t)MK_CT, te - t0) * kTileBytes;
  mbar_arrive_expect_tx(bar, bytes);
  bulk_g2s(stage, p.tiles + (size_t)t0 * kTileBytes, bytes, bar);
  s.ck++;
}

// ---------------------------------------------------------------------------
// GEMV phase: input prologue (all threads) then each warp's share of tiles
struct SmemLayout {
  uint8_t *stages;
  uint64_t *bars;
  uint4 *xzero;
  float *wpart;  // [warps][2][16] partial segments of the current GEMV phase
  uint8_t *u;    // union region
};

CH_DEV void gemv_prologue(const Phase &p, const MegaArgs &a, uint4 *xf, float *vec, float *red) {
  const uint32_t K = p.K, nb = K / 32;
  const bool writer = (blockIdx.x == 0);
  if (p.pm == PM_DIRECT) {
    for (uint32_t b = threadIdx.x; b < nb; b += blockDim.x) {
      float v[32];
      load32(p.x_in + b * 32, v);
      block_to_fragments(v, xf + b * 8);
    }
    return;
  }
  if (p.pm == PM_GELU) {  // act vector finished by the gate|up phase
    for (uint32_t b = threadIdx.x; b < nb; b += blockDim.x) {
      float v[32];
      const float4 *q = reinterpret_cast<const float4 *>(p.r_in.direct + b * 32);
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const float4 f = __ldcg(q + i);
        v[4 * i] = f.x, v[4 * i + 1] = f.y, v[4 * i + 2] = f.z, v[4 * i + 3] = f.w;
      }
      block_to_fragments(v, xf + b * 8);
    }
    return;
  }
  float ss = 0.f;
  if (p.pm == PM_NORM) {
    for (uint32_t b = threadIdx.x; b < nb; b += blockDim.x) {
      float v[32];
      load32(p.x_in + b * 32, v);
#pragma unroll
      for (int e = 0; e < 32; e++) ss = __fmaf_rn(v[e], v[e], ss);
      store32(vec + b * 32, v);
    }
  } else {  // PM_ADD_NORM: r' = post_w ? rmsnorm(r) * post_w : r ; x = (x_in + r') * scalar
    gather_rows(p.r_in, 0, K, vec);
    float inv_r = 1.0f;
    if (p.post_w) {
      float sr = 0.f;
      for (uint32_t i = threadIdx.x; i < K; i += blockDim.x) sr = __fmaf_rn(vec[i], vec[i], sr);
      sr = block_sum(sr, red);
      inv_r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sr, (float)K), a.eps)));
    }
    for (uint32_t b = threadIdx.x; b < nb; b += blockDim.x) {
      float r[32], x[32], w[32];
      load32(vec + b * 32, r);
      load32(p.x_in + b * 32, x);
      if (p.post_w) load32(p.post_w + b * 32, w);
#pragma unroll
      for (int e = 0; e < 32; e++) {
        const float rr = p.post_w ? __fmul_rn(__fmul_rn(r[e], inv_r), w[e]) : r[e];
        x[e] = __fmul_rn(__fadd_rn(x[e], rr), p.scalar);
        ss = __fmaf_rn(x[e], x[e], ss);
      }
      store32(vec + b * 32, x);
      if (writer && p.x_out) store32(p.x_out + b * 32, x);
    }
  }
  ss = block_sum(ss, red);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), a.eps)));
  for (uint32_t b = threadIdx.x; b < nb; b += blockDim.x) {
    float v[32], w[32];
    load32(vec + b * 32, v);
    load32(p.norm_w + b * 32, w);
#pragma unroll
    for (int e = 0; e < 32; e++) v[e] = __fmul_rn(__fmul_rn(v[e], inv), w[e]);
    if (writer && p.normed_out) store32(p.normed_out + b * 32, v);
    block_to_fragments(v, xf + b * 8);
  }
}

// After every warp of the CTA finished its tiles: fold the warps' partial segments.
// Row tiles inside the CTA's range go to `direct`, straddling ones to the CTA's slot.
CH_DEV void cta_combine(const Phase &p, const float *wpart) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t c = blockIdx.x, KT = p.k_tiles;
  const uint32_t cb = cta_begin(p.out, c), ce = cta_begin(p.out, c + 1);
  if (ce == cb) return;
  const uint32_t rt0 = cb / KT, rt1 = (ce - 1) / KT;
  for (uint32_t rt = rt0 + warp; rt <= rt1; rt += MK_NW) {
    const uint32_t t_lo = rt * KT, t_hi = t_lo + KT - 1;
    const uint32_t a_lo = max(t_lo, cb), a_hi = min(t_hi, ce - 1);
    const uint32_t w0 = part_warp_of(a_lo, p.q, p.rem), w1 = part_warp_of(a_hi, p.q, p.rem);
    const bool inside = cb <= t_lo && t_hi < ce;
    if (w0 == w1 && inside) continue;  // one warp covered the whole row tile: already direct
    float sum = 0.f;
    if (lane < 16)
      for (uint32_t w = w0; w <= w1; w++) {
        const uint32_t slot = part_begin(w, p.q, p.rem) < t_lo ? 1u : 0u;
        sum = __fadd_rn(sum, wpart[((w - c * MK_NW) * 2 + slot) * 16 + lane]);
      }
    const float up = __shfl_down_sync(0xffffffffu, sum, 8);
    if (inside) {
      if (p.out.act) {
        if (lane < 8) p.out.direct[rt * 8 + lane] = __fmul_rn(gelu_tanh(sum), up);
      } else if (lane < 16) {
        p.out.direct[rt * 16 + lane] = sum;
      }
    } else {
      // straddling row tile: publish this CTA's sum; the last CTA to arrive finishes it
      const uint32_t slot = cb < t_lo ? 1u : 0u;
      if (lane < 16) p.out.partial[((size_t)c * 2 + slot) * 16 + lane] = sum;
      __threadfence();
      __syncwarp();
      uint32_t old = 0;
      if (lane == 0) old = atomicAdd(&p.out.counters[rt], 1u);
      old = __shfl_sync(0xffffffffu, old, 0);
      const uint32_t c0 = cta_of(p.out, t_lo), c1 = cta_of(p.out, t_hi);
      if (old == c1 - c0) {
        __threadfence();
        float tot = 0.f;
        if (lane < 16)
          for (uint32_t cc = c0; cc <= c1; cc++) {
            const uint32_t sl = cta_begin(p.out, cc) < t_lo ? 1u : 0u;
            tot = __fadd_rn(tot, __ldcg(&p.out.partial[((size_t)cc * 2 + sl) * 16 + lane]));
          }
        const float tup = __shfl_down_sync(0xffffffffu, tot, 8);
        if (p.out.act) {
          if (lane < 8) p.out.direct[rt * 8 + lane] = __fmul_rn(gelu_tanh(tot), tup);
        } else if (lane < 16) {
          p.out.direct[rt * 16 + lane] = tot;
        }
        if (lane == 0) p.out.counters[rt] = 0u;
      }
    }
  }
}

template <int FMT>
CH_DEV void gemv_tiles(const Phase &p, const MegaArgs &a, uint32_t gw, const SmemLayout &L, const uint4 *xf,
                       uint32_t &cidx, Stream &st, bool &ok) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  uint8_t *my_stages = L.stages + (size_t)warp * MK_SPW * MK_STAGE;
  uint64_t *my_bars = L.bars + warp * MK_SPW;
  const uint32_t KT = p.k_tiles;
  const uint32_t tb = part_begin(gw, p.q, p.rem), te = part_begin(gw + 1, p.q, p.rem);
  const uint32_t nchunks = (te - tb + MK_CT - 1) / MK_CT;
  const uint4 *xb = (g < 2) ? xf + t * 2 + g : L.xzero;
  const uint32_t xs = (g < 2) ? 8u : 0u;
  uint32_t rt = tb / KT, kt = tb - (tb / KT) * KT, cur_rt = 0xFFFFFFFFu, kt_begin = 0;
  float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
  bool first_seg = true;
  auto flush = [&](uint32_t frt, uint32_t kb, uint32_t ke) {
    const float acc0 = __fadd_rn(a0, b0), acc1 = __fadd_rn(a1, b1);
    if (t == 0) {
      if (kb == 0 && ke == KT) {
        if (p.out.act) {
          p.out.direct[frt * 8 + g] = __fmul_rn(gelu_tanh(acc0), acc1);
        } else {
          p.out.direct[frt * 16 + g] = acc0;
          p.out.direct[frt * 16 + g + 8] = acc1;
        }
      } else {
        const uint32_t slot = first_seg ? 0u : 1u;
        L.wpart[(warp * 2 + slot) * 16 + g] = acc0;
        L.wpart[(warp * 2 + slot) * 16 + g + 8] = acc1;
      }
    }
    first_seg = false;
  };
  for (uint32_t j = 0; j < nchunks; j++) {
    const uint32_t s = cidx % MK_SPW;
    if (ok && !mbar_wait_bounded(&my_bars[s], (cidx / MK_SPW) & 1, a.err)) ok = false;
    const uint8_t *stg = my_stages + (size_t)s * MK_STAGE;
    const uint32_t t0 = tb + j * MK_CT;
    const uint32_t nt = min((uint32_t)MK_CT, te - t0);
    uint32_t i = 0;
    while (i < nt) {
      if (rt != cur_rt) {
        if (cur_rt != 0xFFFFFFFFu) flush(cur_rt, kt_begin, KT);
        cur_rt = rt;
        kt_begin = kt;
        a0 = a1 = b0 = b1 = 0.f;
      }
      const uint32_t run = min(nt - i, KT - kt);
      const uint8_t *pp = stg + (size_t)i * kTileBytes;
      uint32_t r = 0;
      if (run == MK_CT) {
#pragma unroll
        for (int q = 0; q < MK_CT; q += 2) {
          tile_mma<FMT>(pp + q * kTileBytes, kt + q, xb, xs, lane, a0, a1);
          tile_mma<FMT>(pp + (q + 1) * kTileBytes, kt + q + 1, xb, xs, lane, b0, b1);
        }
        r = MK_CT;
      } else {
        for (; r + 2 <= run; r += 2) {
          tile_mma<FMT>(pp + r * kTileBytes, kt + r, xb, xs, lane, a0, a1);
          tile_mma<FMT>(pp + (r + 1) * kTileBytes, kt + r + 1, xb, xs, lane, b0, b1);
        }
        if (r < run) tile_mma<FMT>(pp + r * kTileBytes, kt + r, xb, xs, lane, a0, a1);
      }
      i += run;
      kt += run;
      if (kt == KT) {
        kt = 0;
        rt++;
      }
    }
    __syncwarp();
    cidx++;
    if (lane == 0 && stream_next(a, gw, st)) {
      fence_proxy_async();
      stream_issue(a, gw, st, my_stages + (size_t)s * MK_STAGE, &my_bars[s]);
    }
    __syncwarp();
  }
  if (cur_rt != 0xFFFFFFFFu) flush(cur_rt, kt_begin, te - cur_rt * KT);
}

// ---------------------------------------------------------------------------
// ATTN phase: work item (kv head, slot chunk) per CTA; qkv_rope.wgsl + decode_attn.wgsl
template <int R>
CH_DEV void attn_phase(const Phase &p, const MegaArgs &a, uint8_t *u, float *red) {
  constexpr int D = 256, EPL = 8;
  constexpr int PVW = (R <= 2) ? MK_NW : (MK_NW * 2 / R);  // warps accumulating P*V (bounds smem)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const StepParams sp = *a.sp;
  const uint32_t S = p.is_sliding ? sp.n_sliding : sp.n_active;
  const uint32_t *list = p.is_sliding ? sp.sliding : sp.active;
  const uint32_t max_splits = a.attn_max_splits;
  const uint32_t chunk = max(kMinChunk, (S + max_splits - 1) / max_splits);
  const uint32_t nsplit = S == 0 ? 1u : (S + chunk - 1) / chunk;
  const uint32_t item = blockIdx.x;
  if (item >= a.nkv * nsplit) return;
  const uint32_t kvh = item / nsplit, split = item % nsplit;
  const uint32_t c0 = split * chunk, c1 = min(S, c0 + chunk), n = c1 > c0 ? c1 - c0 : 0;
  const size_t kv_dim = (size_t)a.nkv * D;
  const uint32_t chunk_cap = max(kMinChunk, (a.cache_slots + max_splits - 1) / max_splits);

  float *raw = reinterpret_cast<float *>(u);   // [R+2][D]
  float *q_s = raw, *k_new = raw + R * D, *v_new = k_new + D;
  float *o_s = v_new + D;                      // [PVW][R][D]
  float *sc = o_s + PVW * R * D;               // [R][chunk_cap]
  float *cmb = sc + R * chunk_cap;             // [R][max_splits]
  float *stat = cmb + R * max_splits;          // [2R]

  // prefetch this CTA's K/V rows toward L2 while the heads are assembled
  for (uint32_t i = c0 + tid; i < c1; i += MK_THREADS) {
    const uint32_t phys = list[i];
    if (phys < a.cache_slots) {
      const __half *kr = p.k_cache + (size_t)phys * kv_dim + (size_t)kvh * D;
      const __half *vr = p.v_cache + (size_t)phys * kv_dim + (size_t)kvh * D;
      asm volatile("prefetch.global.L2 [%0];" ::"l"(kr));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(kr + 128));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(vr));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(vr + 128));
    }
  }
  // raw q heads | k | v rows of this kv head from the q|k|v GEMV output
  gather_rows(p.r_in, kvh * R * D, (kvh + 1) * R * D, raw);
  gather_rows(p.r_in, a.nq * D + kvh * D, a.nq * D + (kvh + 1) * D, k_new);
  gather_rows(p.r_in, a.nq * D + (uint32_t)kv_dim + kvh * D, a.nq * D + (uint32_t)kv_dim + (kvh + 1) * D, v_new);
  for (int h = warp; h < R + 2; h += MK_NW) {
    float *hd = raw + h * D;
    if (h <= R)
      head_norm_rope_s(hd, h < R ? p.q_norm_w : p.k_norm_w, hd, D, a.rot, p.rope_cs, a.eps, true, lane);
    else
      head_norm_rope_s(hd, nullptr, hd, D, a.rot, nullptr, a.eps, false, lane);
    __syncwarp();
    if (h >= R) {  // f16 cache row of the new K / V, written by split 0
      __half *dst = (h == R ? p.k_cache : p.v_cache) + (size_t)sp.slot * kv_dim + (size_t)kvh * D;
      for (uint32_t d = lane; d < D; d += 32) {
        const __half hv = __float2half_rn(hd[d]);
        hd[d] = __half2float(hv);
        if (split == 0 && sp.slot < a.cache_slots) dst[d] = hv;
      }
    }
  }
  if (split == 0 && sp.slot >= a.cache_slots && tid == 0) atomicOr(a.err, DEV_ERR_BAD_SLOT);
  __syncthreads();

  // scores
  float qr[R][EPL];
#pragma unroll
  for (int h = 0; h < R; h++)
#pragma unroll
    for (int e = 0; e < EPL; e++) qr[h][e] = q_s[h * D + lane * EPL + e];
  for (uint32_t i = warp; i < n; i += MK_NW) {
    const uint32_t phys = list[c0 + i];
    float kv[EPL];
    bool valid = true;
    if (phys == sp.slot) {
#pragma unroll
      for (int e = 0; e < EPL; e++) kv[e] = k_new[lane * EPL + e];
    } else if (phys < a.cache_slots) {
      const uint4 rw = *reinterpret_cast<const uint4 *>(p.k_cache + (size_t)phys * kv_dim + (size_t)kvh * D + lane * EPL);
      const __half2 *hp = reinterpret_cast<const __half2 *>(&rw);
#pragma unroll
      for (int e = 0; e < EPL / 2; e++) {
        const float2 f = __half22float2(hp[e]);
        kv[2 * e] = f.x;
        kv[2 * e + 1] = f.y;
      }
    } else {
      valid = false;
#pragma unroll
      for (int e = 0; e < EPL; e++) kv[e] = 0.f;
    }
#pragma unroll
    for (int h = 0; h < R; h++) {
      float dot = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; e++) dot = __fmaf_rn(qr[h][e], kv[e], dot);
      dot = warp_sum(dot);
      if (lane == 0) sc[h * chunk_cap + i] = valid ? __fmul_rn(dot, p.attn_scale) : -INFINITY;
    }
    if (!valid && lane == 0) atomicOr(a.err, DEV_ERR_BAD_LIST);
  }
  __syncthreads();
  for (int h = warp; h < R; h += MK_NW) {
    float m = -1e9f;  // decode_attn.wgsl:261
    for (uint32_t i = lane; i < n; i += 32) m = fmaxf(m, sc[h * chunk_cap + i]);
    m = warp_max(m);
    float l = 0.f;
    for (uint32_t i = lane; i < n; i += 32) {
      const float e = expf(__fsub_rn(sc[h * chunk_cap + i], m));
      sc[h * chunk_cap + i] = e;
      l = __fadd_rn(l, e);
    }
    l = warp_sum(l);
    if (lane == 0) {
      stat[2 * h] = m;
      stat[2 * h + 1] = l;
    }
  }
  __syncthreads();
  // weighted V (PVW warps)
  if (warp < PVW) {
    float acc[R][EPL];
#pragma unroll
    for (int h = 0; h < R; h++)
#pragma unroll
      for (int e = 0; e < EPL; e++) acc[h][e] = 0.f;
    for (uint32_t i = warp; i < n; i += PVW) {
      const uint32_t phys = list[c0 + i];
      float vv[EPL];
      if (phys == sp.slot) {
#pragma unroll
        for (int e = 0; e < EPL; e++) vv[e] = v_new[lane * EPL + e];
      } else if (phys < a.cache_slots) {
        const uint4 rw =
            *reinterpret_cast<const uint4 *>(p.v_cache + (size_t)phys * kv_dim + (size_t)kvh * D + lane * EPL);
        const __half2 *hp = reinterpret_cast<const __half2 *>(&rw);
#pragma unroll
        for (int e = 0; e < EPL / 2; e++) {
          const float2 f = __half22float2(hp[e]);
          vv[2 * e] = f.x;
          vv[2 * e + 1] = f.y;
        }
      } else {
#pragma unroll
        for (int e = 0; e < EPL; e++) vv[e] = 0.f;
      }
#pragma unroll
      for (int h = 0; h < R; h++) {
        const float pr = sc[h * chunk_cap + i];
#pragma unroll
        for (int e = 0; e < EPL; e++) acc[h][e] = __fmaf_rn(pr, vv[e], acc[h][e]);
      }
    }
#pragma unroll
    for (int h = 0; h < R; h++)
#pragma unroll
      for (int e = 0; e < EPL; e++) o_s[(warp * R + h) * D + lane * EPL + e] = acc[h][e];
  }
  __syncthreads();
  float *part = a.attn_partial + ((size_t)(kvh * max_splits + split) * R) * (D + 2);
  for (int idx = tid; idx < R * D; idx += MK_THREADS) {
    const int h = idx / D, d = idx % D;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < PVW; w++) s = __fadd_rn(s, o_s[(w * R + h) * D + d]);
    part[h * (D + 2) + d] = s;
  }
  if (tid < R) {
    part[tid * (D + 2) + D] = stat[2 * tid];
    part[tid * (D + 2) + D + 1] = stat[2 * tid + 1];
  }
  __threadfence();
  __syncthreads();
  __shared__ uint32_t last_flag;
  if (tid == 0) last_flag = (atomicAdd(&a.attn_counters[kvh], 1u) == nsplit - 1) ? 1u : 0u;
  __syncthreads();
  if (!last_flag) return;
  __threadfence();
  const float *base = a.attn_partial + ((size_t)kvh * max_splits * R) * (D + 2);
  for (int idx = tid; idx < R * (int)nsplit; idx += MK_THREADS) {
    const int h = idx / nsplit, j = idx % nsplit;
    cmb[h * max_splits + j] = __ldcg(&base[((size_t)j * R + h) * (D + 2) + D]);
  }
  __syncthreads();
  if (tid < R) {
    float M = -INFINITY, Lsum = 0.f;
    for (uint32_t j = 0; j < nsplit; j++) M = fmaxf(M, cmb[tid * max_splits + j]);
    for (uint32_t j = 0; j < nsplit; j++) {
      const float f = expf(__fsub_rn(cmb[tid * max_splits + j], M));
      Lsum = __fmaf_rn(__ldcg(&base[((size_t)j * R + tid) * (D + 2) + D + 1]), f, Lsum);
      cmb[tid * max_splits + j] = f;
    }
    stat[2 * tid] = __fdiv_rn(1.0f, __fadd_rn(Lsum, 1e-9f));
  }
  __syncthreads();
  for (int idx = tid; idx < R * D; idx += MK_THREADS) {
    const int h = idx / D, d = idx % D;
    float O = 0.f;
    for (uint32_t j = 0; j < nsplit; j++)
      O = __fmaf_rn(__ldcg(&base[((size_t)j * R + h) * (D + 2) + d]), cmb[h * max_splits + j], O);
    p.attn_out[(size_t)(kvh * R + h) * D + d] = __fmul_rn(O, stat[2 * h]);
  }
  if (tid == 0) a.attn_counters[kvh] = 0u;
}

// ---------------------------------------------------------------------------
// TOPK phase: each CTA selects the top 64 of its vocab slice, last CTA merges
CH_DEV void topk_phase(const Phase &p, const MegaArgs &a, uint8_t *u) {
  constexpr int E1 = 8, E2 = 20;  // per-thread keys: slice <= 4096, candidates <= 10240
  uint32_t *hist = reinterpret_cast<uint32_t *>(u);
  uint32_t *sh = hist + 256;
  uint32_t *cnt = sh + 4;
  uint64_t *buf = reinterpret_cast<uint64_t *>(cnt + 4);
  uint64_t *sorted = buf + 64;
  float *lg = reinterpret_cast<float *>(sorted + 64);  // this CTA's slice of the logits
  __shared__ uint32_t last_flag;
  const int tid = threadIdx.x;
  const uint32_t G = gridDim.x, V = p.vocab;
  const uint32_t lo = (uint32_t)(((uint64_t)V * blockIdx.x) / G), hi = (uint32_t)(((uint64_t)V * (blockIdx.x + 1)) / G);
  gather_rows(p.r_in, lo, hi, lg);
  {
    uint64_t k[E1];
#pragma unroll
    for (int e = 0; e < E1; e++) {
      const uint32_t idx = lo + e * MK_THREADS + tid;
      if (idx < hi) {
        const float v = softcap(lg[idx - lo]);
        k[e] = ((uint64_t)sortable(v) << 32) | (uint64_t)(0xFFFFFFFFu - idx);
      } else {
        k[e] = 0;
      }
    }
    const uint64_t thr = block_kth_largest<E1>(k, 64, hist, sh);
    collect_sorted64<E1>(k, thr, buf, cnt, sorted);
    if (tid < 64) a.topk_cand[(size_t)blockIdx.x * 64 + tid] = sorted[tid];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) last_flag = (atomicAdd(a.topk_counter, 1u) == G - 1) ? 1u : 0u;
  __syncthreads();
  if (!last_flag) return;
  __threadfence();
  uint64_t k[E2];
  const uint32_t ncand = G * 64;
#pragma unroll
  for (int e = 0; e < E2; e++) {
    const uint32_t i = e * MK_THREADS + tid;
    k[e] = i < ncand ? __ldcg(&a.topk_cand[i]) : 0ull;
  }
  const uint64_t thr = block_kth_largest<E2>(k, 64, hist, sh);
  collect_sorted64<E2>(k, thr, buf, cnt, sorted);
  if (tid < 64) {
    const uint64_t key = sorted[tid];
    uint32_t id = 0;
    float val = -1e30f;
    if (key != 0) {
      id = 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFu);
      val = unsortable((uint32_t)(key >> 32));
    }
    a.ids[tid] = id;
    a.vals[tid] = val;
    if (tid == 0) {
      if (a.token_out) *a.token_out = id;
      if (a.sp_rw) {
        const uint32_t step = a.sp_rw->step;
        if (a.token_hist && step < a.hist_cap) a.token_hist[step] = id;
        a.sp_rw->step = step + 1;
      }
    }
  }
  if (tid == 0) *a.topk_counter = 0u;
}

// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(MK_THREADS, 1) decode_step_kernel(const MegaArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  SmemLayout L;
  L.stages = smem;
  L.bars = reinterpret_cast<uint64_t *>(smem + MK_NW * MK_SPW * MK_STAGE);
  L.xzero = reinterpret_cast<uint4 *>(smem + MK_NW * MK_SPW * MK_STAGE + MK_NW * MK_SPW * 8);
  L.wpart = reinterpret_cast<float *>(L.xzero + 1);
  L.u = reinterpret_cast<uint8_t *>(L.wpart + MK_NW * 2 * 16);
  __shared__ float red[32];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t gw = blockIdx.x * MK_NW + warp;
  uint8_t *my_stages = L.stages + (size_t)warp * MK_SPW * MK_STAGE;
  uint64_t *my_bars = L.bars + warp * MK_SPW;
  Stream st{0, 0};
  if (lane == 0) {
    for (int s = 0; s < MK_SPW; s++) mbar_init(&my_bars[s], 1);
    fence_mbar_init();
    for (int s = 0; s < MK_SPW; s++)
      if (stream_next(a, gw, st)) stream_issue(a, gw, st, my_stages + (size_t)s * MK_STAGE, &my_bars[s]);
  }
  if (threadIdx.x == 0) *L.xzero = make_uint4(0u, 0u, 0u, 0u);
  // every lane keeps the stream cursor (lane 0's copy drives the issues)
  st.ph = __shfl_sync(0xffffffffu, st.ph, 0);
  st.ck = __shfl_sync(0xffffffffu, st.ck, 0);
  __syncthreads();

  const unsigned long long epoch = *a.epoch;
  const unsigned long long base = epoch * (unsigned long long)(a.nphases - 1) * gridDim.x;
  uint32_t cidx = 0;
  bool ok = true;
  for (uint32_t pi = 0; pi < a.nphases; pi++) {
    const Phase &p = a.phases[pi];
    if (p.kind == PH_GEMV) {
      uint4 *xf = reinterpret_cast<uint4 *>(L.u);
      float *vec = reinterpret_cast<float *>(xf + (p.K / 32) * 8);
      gemv_prologue(p, a, xf, vec, red);
      __syncthreads();
      if (p.fmt == FMT_Q4)
        gemv_tiles<FMT_Q4>(p, a, gw, L, xf, cidx, st, ok);
      else
        gemv_tiles<FMT_Q8>(p, a, gw, L, xf, cidx, st, ok);
      __syncthreads();
      cta_combine(p, L.wpart);
    } else if (p.kind == PH_ATTN) {
      switch (a.nq / a.nkv) {
        case 1: attn_phase<1>(p, a, L.u, red); break;
        case 2: attn_phase<2>(p, a, L.u, red); break;
        default: attn_phase<4>(p, a, L.u, red); break;
      }
    } else {
      topk_phase(p, a, L.u);
    }
    if (pi + 1 < a.nphases) grid_barrier(a.arrive, base + (unsigned long long)(pi + 1) * gridDim.x, a.err);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) *a.epoch = (uint32_t)(epoch + 1);
}

size_t mk_smem_bytes(uint32_t max_k, uint32_t hidden, uint32_t ratio, uint32_t max_splits, uint32_t cache_slots) {
  const size_t fixed = (size_t)MK_NW * MK_SPW * MK_STAGE + MK_NW * MK_SPW * 8 + 16 + MK_NW * 2 * 16 * 4;
  // xf (K*4 bytes) + vec (kVecRows floats; the norm prologues need hidden <= kVecRows)
  const size_t gemv = (size_t)max_k * 4 + (size_t)std::max(hidden, kVecRows) * 4;
  const uint32_t pvw = ratio <= 2 ? MK_NW : MK_NW * 2 / ratio;
  const uint32_t chunk_cap = std::max(kMinChunk, (cache_slots + max_splits - 1) / max_splits);
  const size_t attn = 4 * ((size_t)(ratio + 2) * 256 + (size_t)pvw * ratio * 256 + (size_t)ratio * chunk_cap +
                           (size_t)ratio * max_splits + 2 * ratio);
  const size_t topk = 256 * 4 + 32 + 128 * 8 + 4096 * 4;
  return fixed + std::max({gemv, attn, topk});
}

cudaError_t launch_decode_step(const MegaArgs &a, size_t smem, cudaStream_t s) {
  static size_t attr = 0;
  if (smem > attr) {
    cudaError_t e = cudaFuncSetAttribute(decode_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.grid);
  cfg.blockDim = dim3(MK_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr_c[1];
  attr_c[0].id = cudaLaunchAttributeCooperative;
  attr_c[0].val.cooperative = 1;
  cfg.attrs = attr_c;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_step_kernel, a);
}

}  // namespace ch
