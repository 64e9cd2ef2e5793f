// attention.cu -- decode attention over the 4,096-slot ring-buffer KV cache.
//
// Restates, in one kernel, the reference's two decode passes:
//   qkv_rope.wgsl:25-180   per-head RMSNorm * q_norm / k_norm, half-split RoPE at
//                          `clock`, V unit-RMSNorm, K/V written to cache[slot]
//   decode_attn.wgsl:24-218 scores = q.k * scale over the slot list, softmax
//                          (max seeded at -1e9, 1/(sum + 1e-9)), weighted V; GQA
//                          kv_head = q_head / ratio
// B200 design: split-K over the slot list (flash-decode).  Grid = kv_heads x
// splits; each CTA owns every q head of its kv head (GQA packing), recomputes
// the tiny norm + RoPE of q/k/v for that head itself (so no separate launch),
// streams its slice of the gathered f16 K/V rows with 16-byte loads, keeps
// per-chunk max / sum / weighted V, and the last CTA of each kv head combines
// the chunk partials in fixed order (deterministic).  The split count adapts to
// the list length (>= 64 slots per CTA).  The fresh K/V of the current slot are
// used from shared memory, so no CTA reads a cache row that another CTA of the
// same launch is writing.  RoPE (cos, sin) for the step's clock come from a
// table computed once per step (double precision, rounded once).
#include <algorithm>

#include "common.cuh"
#include "core.cuh"
#include "kernels.cuh"

namespace ch {

namespace {
constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kMaxRatio = 8;
}  // namespace

int attn_default_splits(uint32_t nkv) {
  int target = 2 * num_sms();
  int s = (int)((target + nkv - 1) / nkv);
  if (s < 1) s = 1;
  if (s > 64) s = 64;
  return s;
}
size_t attn_partial_floats(uint32_t nkv, uint32_t ratio, uint32_t D, int splits) {
  return (size_t)nkv * splits * ratio * (D + 2);
}

namespace {
constexpr uint32_t kMinChunk = 64;  // slots per CTA before splitting further stops paying
}

template <int R>
__global__ void __launch_bounds__(kAttnThreads) decode_attn_kernel(const AttnArgs a, int max_splits, int chunk_cap) {
  constexpr int D = 256, EPL = D / 32;  // elements per lane
  extern __shared__ __align__(16) float sm[];
  float *raw = sm;                        // [R+2][D] staged raw q heads | k | v
  float *q_s = raw;                       // normalized in place: [R][D]
  float *k_new = raw + R * D;             // [D]
  float *v_new = k_new + D;               // [D]
  float *o_s = v_new + D;                 // [warps][R][D]
  float *sc = o_s + kAttnWarps * R * D;   // [R][chunk_cap]
  float *cmb = sc + R * chunk_cap;        // [R][max_splits] combine factors
  uint32_t *slist = reinterpret_cast<uint32_t *>(cmb + R * max_splits);  // [chunk_cap] this chunk's slots
  __shared__ float stat[2 * kMaxRatio];
  __shared__ uint32_t last_flag;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t kvh = blockIdx.x, split = blockIdx.y, b = blockIdx.z;
  const size_t kv_dim = (size_t)a.nkv * D;
  // this token's views (batched decode: one token per stream)
  const float *qkv = a.qkv + (size_t)b * a.qkv_stride;
  const float2 *rope_cs = a.rope_cs + (size_t)b * a.rope_stride;
  const size_t coff = a.stream ? (size_t)a.stream[b] * a.cache_stride : 0;
  __half *k_cache = a.k_cache + coff, *v_cache = a.v_cache + coff;
  float *out = a.out + (size_t)b * a.out_stride;
  float *partial = a.partial + (size_t)b * a.nkv * max_splits * R * (D + 2);
  uint32_t *counters = a.counters + (size_t)b * a.nkv;

  // step state was written before the previous kernel started (see model.cu)
  const StepParams sp = a.sp[b];
  const uint32_t S = a.is_sliding ? sp.n_sliding : sp.n_active;
  const uint32_t *list = a.is_sliding ? sp.sliding : sp.active;
  // adaptive split: at least kMinChunk slots per CTA, at most max_splits CTAs per kv head
  const uint32_t chunk = max(kMinChunk, (S + max_splits - 1) / (uint32_t)max_splits);
  const uint32_t nsplit = S == 0 ? 1u : (S + chunk - 1) / chunk;
  if (split >= nsplit) return;  // idle CTA (exits count as the PDL trigger)
  const uint32_t c0 = split * chunk, c1 = min(S, c0 + chunk);
  const uint32_t n = c1 > c0 ? c1 - c0 : 0;

  // stage this chunk's slot list (the row loads below then wait for one round trip, not
  // two); for a single token also warm L2 with the chunk's K/V rows while the
  // projections finish -- a batch's rows (hundreds of MB per layer) would not stay there
  for (uint32_t i = tid; i < n; i += kAttnThreads) {
    const uint32_t phys = list[c0 + i];
    slist[i] = phys;
    if (a.n_tok == 1 && phys < a.cache_slots) {
      const __half *kr = k_cache + (size_t)phys * kv_dim + (size_t)kvh * D;
      const __half *vr = v_cache + (size_t)phys * kv_dim + (size_t)kvh * D;
      asm volatile("prefetch.global.L2 [%0];" ::"l"(kr));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(kr + 128));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(vr));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(vr + 128));
    }
  }
  grid_dep_wait();

  // ---- stage q heads | k | v of this kv head (one round trip), then norm + rope ----
  const float *kraw = qkv + (size_t)a.nq * D;
  for (int idx = tid; idx < (R + 2) * (D / 4); idx += kAttnThreads) {
    const int h = idx / (D / 4), f = idx % (D / 4);
    const float *src = h < R ? qkv + (size_t)(kvh * R + h) * D : (h == R ? kraw : kraw + kv_dim) + (size_t)kvh * D;
    reinterpret_cast<float4 *>(raw + h * D)[f] = reinterpret_cast<const float4 *>(src)[f];
  }
  __syncthreads();
  for (int h = warp; h < R + 2; h += kAttnWarps) {
    float *hd = raw + h * D;
    if (h <= R) {
      head_norm_rope_s(hd, h < R ? a.q_norm_w : a.k_norm_w, hd, D, a.rot, rope_cs, a.eps, true, lane);
    } else {
      head_norm_rope_s(hd, nullptr, hd, D, a.rot, nullptr, a.eps, false, lane);
    }
    __syncwarp();
    if (h >= R) {  // round the new K / V to the cache's f16 and write them (split 0 only)
      __half *dst = (h == R ? k_cache : v_cache) + (size_t)sp.slot * kv_dim + (size_t)kvh * D;
      for (uint32_t d = lane; d < D; d += 32) {
        const __half hv = __float2half_rn(hd[d]);
        hd[d] = __half2float(hv);
        if (split == 0 && sp.slot < a.cache_slots) dst[d] = hv;
      }
    }
  }
  if (split == 0 && sp.slot >= a.cache_slots && tid == 0) atomicOr(a.err, DEV_ERR_BAD_SLOT);
  __syncthreads();
  grid_dep_launch();

  // ---- scores: one slot per warp iteration, lane owns dims [lane*8, lane*8+8) ----
  float qr[R][EPL];
#pragma unroll
  for (int h = 0; h < R; h++)
#pragma unroll
    for (int e = 0; e < EPL; e++) qr[h][e] = q_s[h * D + lane * EPL + e];

  // rows of this chunk, kU slots per warp iteration with every load issued before any is
  // used (one slot per iteration left each warp waiting a full memory round trip per
  // slot); the per-slot arithmetic and the per-warp slot order are unchanged.
  // kind: 0 = cache row in rw, 1 = the new row (shared memory), 2 = invalid slot, 3 = past n
  constexpr int kU = 4;
  auto fetch = [&](const __half *cache, uint32_t i, uint4 &rw) -> int {
    if (i >= n) return 3;
    const uint32_t phys = slist[i];
    if (phys == sp.slot) return 1;
    if (phys >= a.cache_slots) return 2;
    rw = *reinterpret_cast<const uint4 *>(cache + (size_t)phys * kv_dim + (size_t)kvh * D + lane * EPL);
    return 0;
  };
  auto unpack = [&](int kind, const uint4 &rw, const float *fresh, float (&f)[EPL]) {
    if (kind == 1) {
#pragma unroll
      for (int e = 0; e < EPL; e++) f[e] = fresh[lane * EPL + e];
    } else if (kind == 0) {
      const __half2 *hp = reinterpret_cast<const __half2 *>(&rw);
#pragma unroll
      for (int e = 0; e < EPL / 2; e++) {
        const float2 v = __half22float2(hp[e]);
        f[2 * e] = v.x;
        f[2 * e + 1] = v.y;
      }
    } else {
#pragma unroll
      for (int e = 0; e < EPL; e++) f[e] = 0.f;
    }
  };
  for (uint32_t i0 = warp; i0 < n; i0 += kU * kAttnWarps) {
    uint4 rw[kU];
    int kind[kU];
#pragma unroll
    for (int u = 0; u < kU; u++) kind[u] = fetch(k_cache, i0 + u * kAttnWarps, rw[u]);
#pragma unroll
    for (int u = 0; u < kU; u++) {
      if (kind[u] == 3) continue;
      const uint32_t i = i0 + u * kAttnWarps;
      float kv[EPL];
      unpack(kind[u], rw[u], k_new, kv);
      const bool valid = kind[u] != 2;
#pragma unroll
      for (int h = 0; h < R; h++) {
        float dot = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; e++) dot = __fmaf_rn(qr[h][e], kv[e], dot);
        dot = warp_sum(dot);
        if (lane == 0) sc[h * chunk_cap + i] = valid ? __fmul_rn(dot, a.scale) : -INFINITY;
      }
      if (!valid && lane == 0) atomicOr(a.err, DEV_ERR_BAD_LIST);
    }
  }
  __syncthreads();

  // ---- chunk max / exp / sum per q head (warp h handles head h) ----
  for (int h = warp; h < R; h += kAttnWarps) {
    float m = -1e9f;  // decode_attn.wgsl:81
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

  // ---- weighted V ----
  float acc[R][EPL];
#pragma unroll
  for (int h = 0; h < R; h++)
#pragma unroll
    for (int e = 0; e < EPL; e++) acc[h][e] = 0.f;
  for (uint32_t i0 = warp; i0 < n; i0 += kU * kAttnWarps) {
    uint4 rw[kU];
    int kind[kU];
#pragma unroll
    for (int u = 0; u < kU; u++) kind[u] = fetch(v_cache, i0 + u * kAttnWarps, rw[u]);
#pragma unroll
    for (int u = 0; u < kU; u++) {
      if (kind[u] == 3) continue;
      const uint32_t i = i0 + u * kAttnWarps;
      float vv[EPL];
      unpack(kind[u], rw[u], v_new, vv);
#pragma unroll
      for (int h = 0; h < R; h++) {
        const float p = sc[h * chunk_cap + i];
#pragma unroll
        for (int e = 0; e < EPL; e++) acc[h][e] = __fmaf_rn(p, vv[e], acc[h][e]);
      }
    }
  }
#pragma unroll
  for (int h = 0; h < R; h++)
#pragma unroll
    for (int e = 0; e < EPL; e++) o_s[(warp * R + h) * D + lane * EPL + e] = acc[h][e];
  __syncthreads();

  // ---- partial out: [kvh][split][h] = {o[D], m, l} ----
  float *part = partial + ((size_t)(kvh * max_splits + split) * R) * (D + 2);
  for (int idx = tid; idx < R * D; idx += kAttnThreads) {
    const int h = idx / D, d = idx % D;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; w++) s = __fadd_rn(s, o_s[(w * R + h) * D + d]);
    part[h * (D + 2) + d] = s;
  }
  if (tid < R) {
    part[tid * (D + 2) + D] = stat[2 * tid];
    part[tid * (D + 2) + D + 1] = stat[2 * tid + 1];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const uint32_t old = atomicAdd(&counters[kvh], 1u);
    last_flag = (old == nsplit - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (!last_flag) return;
  __threadfence();

  // ---- combine (fixed split order): factors first, then one pipelined pass ----
  const float *base = partial + ((size_t)kvh * max_splits * R) * (D + 2);
  for (int idx = tid; idx < R * (int)nsplit; idx += kAttnThreads) {
    const int h = idx / nsplit, j = idx % nsplit;
    cmb[h * max_splits + j] = __ldcg(&base[((size_t)j * R + h) * (D + 2) + D]);
  }
  __syncthreads();
  if (tid < R) {
    float M = -INFINITY, L = 0.f;
    for (uint32_t j = 0; j < nsplit; j++) M = fmaxf(M, cmb[tid * max_splits + j]);
    for (uint32_t j = 0; j < nsplit; j++) {
      const float f = expf(__fsub_rn(cmb[tid * max_splits + j], M));
      L = __fmaf_rn(__ldcg(&base[((size_t)j * R + tid) * (D + 2) + D + 1]), f, L);
      cmb[tid * max_splits + j] = f;
    }
    stat[2 * tid] = __fdiv_rn(1.0f, __fadd_rn(L, 1e-9f));
  }
  __syncthreads();
  for (int idx = tid; idx < R * D; idx += kAttnThreads) {
    const int h = idx / D, d = idx % D;
    float O = 0.f;
    uint32_t j = 0;
    for (; j + 4 <= nsplit; j += 4) {
      const float p0 = __ldcg(&base[((size_t)(j + 0) * R + h) * (D + 2) + d]);
      const float p1 = __ldcg(&base[((size_t)(j + 1) * R + h) * (D + 2) + d]);
      const float p2 = __ldcg(&base[((size_t)(j + 2) * R + h) * (D + 2) + d]);
      const float p3 = __ldcg(&base[((size_t)(j + 3) * R + h) * (D + 2) + d]);
      O = __fmaf_rn(p0, cmb[h * max_splits + j], O);
      O = __fmaf_rn(p1, cmb[h * max_splits + j + 1], O);
      O = __fmaf_rn(p2, cmb[h * max_splits + j + 2], O);
      O = __fmaf_rn(p3, cmb[h * max_splits + j + 3], O);
    }
    for (; j < nsplit; j++) O = __fmaf_rn(__ldcg(&base[((size_t)j * R + h) * (D + 2) + d]), cmb[h * max_splits + j], O);
    out[(size_t)(kvh * R + h) * D + d] = __fmul_rn(O, stat[2 * h]);
  }
  if (tid == 0) counters[kvh] = 0u;
}

template <int R>
static cudaError_t launch_attn_t(const AttnArgs &a, int splits, cudaStream_t s, bool pdl) {
  const int chunk_cap = (int)std::max<uint32_t>(kMinChunk, (a.cache_slots + splits - 1) / splits);
  const size_t smem = sizeof(float) * ((size_t)(R + 2) * 256 + (size_t)kAttnWarps * R * 256 + (size_t)R * chunk_cap +
                                       (size_t)R * splits) +
                      sizeof(uint32_t) * (size_t)chunk_cap;
  {
    const cudaError_t e = ensure_smem_attr((const void *)decode_attn_kernel<R>, smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.nkv, splits, a.n_tok);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, decode_attn_kernel<R>, a, splits, chunk_cap);
}

cudaError_t launch_decode_attn(const AttnArgs &a, int splits, cudaStream_t s, bool pdl) {
  if (a.D != 256 || a.nkv == 0 || a.nq % a.nkv != 0) return cudaErrorInvalidValue;
  const uint32_t R = a.nq / a.nkv;
  switch (R) {
    case 1: return launch_attn_t<1>(a, splits, s, pdl);
    case 2: return launch_attn_t<2>(a, splits, s, pdl);
    case 4: return launch_attn_t<4>(a, splits, s, pdl);
    case 8: return launch_attn_t<8>(a, splits, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ch
