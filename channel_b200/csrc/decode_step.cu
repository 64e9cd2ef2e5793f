// decode_step.cu -- one greedy decode token as ONE persistent kernel.
//
// Replaces the reference's per-token command buffer of ~12 dispatches per layer
// (src/gpu/model_dispatch.zig:10-45,103-126: fused_qkv_q4, qkv_rope, decode_attn,
// gemv_q4(O), rmsnorm/add_rmsnorm, fused_mlp_q4, gemv_q4(down), ..., gemv_q8 +
// topk_pass1/2) with a phase list executed by a cooperative grid of one CTA per
// SM:
//
//   per layer:  GEMV q|k|v  ->  ATTN  ->  GEMV o  ->  GEMV gate|up  ->  GEMV down
//   tail:       GEMV Q8 LM head  ->  TOPK
//
// B200 design.  A decode token is an HBM weight stream (7.2 GB for the 12B
// shape) with tiny activations in between, so the time that is not weight
// streaming is latency: the dependent steps between two GEMVs.  The kernel is
// built to keep that chain short:
//
//  * Weights never wait for activations.  Every warp owns a balanced share of
//    the tiles of every GEMV phase and streams its shares of ALL phases back to
//    back through its own ring of bulk-copy stages (cp.async.bulk, mbarrier
//    completion, L2 evict-first), so the stream runs on through prologues,
//    attention and barriers.
//  * One grid barrier per phase (a monotonic arrival counter).  A GEMV leaves a
//    row tile that straddles two CTAs as one partial sum per CTA; the consumer
//    adds them up, so producers need no fences or atomics beyond the barrier.
//  * Every activation a phase reads comes into shared memory by bulk copies
//    (the same engine as the weights, so thousands of small loads per SM do not
//    queue behind the weight stream): the inputs that do not depend on the
//    previous phase (residual, norm weights, the attention window's K/V rows,
//    RoPE table) are issued BEFORE the grid barrier, the previous phase's
//    output and its straddle partials right after it -- one copy wait each.
#include <algorithm>

#include "common.cuh"
#include "core.cuh"
#include "decode_step.cuh"

// build-time tuning: stages per warp, tiles per stage
#ifndef CH_MK_SPW
#define CH_MK_SPW 2
#endif
#ifndef CH_MK_CT
#define CH_MK_CT 7
#endif

namespace ch {

namespace {
constexpr int MK_NW = 16;          // warps per CTA (all stream + compute)
constexpr int MK_SPW = CH_MK_SPW;  // bulk-copy stages per warp
// tiles per stage.  The 12B GEMV partitions give each warp n or n + 1 tiles with
// n = 6 (o), 12 (q|k|v), 24 (down), 48 (gate|up) on one GPU and their halves / quarters
// under tensor parallelism; with 7-tile chunks both counts need the same number of
// chunks, so no warp waits for one more bulk-copy round trip than the rest of its phase
// (6-tile chunks: 2.86 ms per token, 7: 2.79 ms).
constexpr int MK_CT = CH_MK_CT;
constexpr int MK_STAGE = MK_CT * kTileBytes;
static_assert(MK_CT >= 2, "a full chunk is consumed in pairs of tiles, plus one when MK_CT is odd");
constexpr int MK_THREADS = MK_NW * 32;
#ifndef CH_MK_MINCHUNK
#define CH_MK_MINCHUNK 32
#endif
constexpr uint32_t kMinChunk = CH_MK_MINCHUNK;  // slots per attention work item before splitting further stops paying
#ifndef CH_MK_WIN
#define CH_MK_WIN 56
#endif
constexpr uint32_t kWinSlots = CH_MK_WIN;  // attention slots per work item staged in shared memory before the barrier
constexpr uint32_t kNoStraddle = 0xFFFFFFFFu;
constexpr int kHeadDim = 256;
constexpr uint32_t kMaxGrid = 255;  // straddle-list entries hold CTA ids in 8 bits
constexpr uint32_t kMaxComb = 24;   // combine items of one CTA and GEMV kind (at most 17 can occur)
}  // namespace

int mk_warps() { return MK_NW; }

// Optional per-phase timeline (build with -DCH_PHASE_TRACE, see bench_phases.py):
// thread 0 of every CTA records %globaltimer at eight points of each phase (marks 0-7),
// lane 0 of warps 0 and 15 at the first chunk and the end of their tiles (marks 8-11),
// and the CTA's SM id once (mark 12 of phase 0).
#ifdef CH_PHASE_TRACE
constexpr int kTraceCtas = 256, kTracePhases = 512, kTraceMarks = 13;  // mark 12: the CTA's SM id
__device__ unsigned long long g_phase_trace[kTraceCtas * kTracePhases * kTraceMarks];
#define PHASE_MARK(pi, k)                                                                               \
  do {                                                                                                  \
    if (threadIdx.x == 0 && blockIdx.x < kTraceCtas && (pi) < kTracePhases)                             \
      g_phase_trace[((size_t)blockIdx.x * kTracePhases + (pi)) * kTraceMarks + (k)] = globaltimer_ns(); \
  } while (0)
// marks 8..11 from lane 0 of warp w inside the tile loop (w = 0: marks 8, 9; w = 15: 10, 11)
#define WARP_MARK(pi, k, w)                                                                             \
  do {                                                                                                  \
    if (threadIdx.x == (w) * 32 && blockIdx.x < kTraceCtas && (pi) < kTracePhases)                      \
      g_phase_trace[((size_t)blockIdx.x * kTracePhases + (pi)) * kTraceMarks + (k)] = globaltimer_ns(); \
  } while (0)
// mark 12 of phase 0: the SM the CTA runs on (%smid)
#define TRACE_SMID()                                                            \
  do {                                                                          \
    if (threadIdx.x == 0 && blockIdx.x < kTraceCtas) {                          \
      uint32_t sm;                                                              \
      asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));                           \
      g_phase_trace[(size_t)blockIdx.x * kTracePhases * kTraceMarks + 12] = sm; \
    }                                                                           \
  } while (0)
#else
#define TRACE_SMID() \
  do {               \
  } while (0)
#define PHASE_MARK(pi, k) \
  do {                    \
  } while (0)
#define WARP_MARK(pi, k, w) \
  do {                      \
  } while (0)
#endif

// ---------------------------------------------------------------------------
// balanced partition of T tiles over GW warps: warp w owns [w*q + min(w,rem), ...)
CH_DEV uint32_t part_begin(uint32_t w, uint32_t q, uint32_t rem) { return w * q + min(w, rem); }
CH_DEV uint32_t part_warp_of(uint32_t t, uint32_t q, uint32_t rem) {
  const uint32_t big = rem * (q + 1);
  return t < big ? t / (q + 1) : rem + (t - big) / q;
}
// CTA c owns tiles [cta_begin(c), cta_begin(c+1)) (stream-K or whole row tiles)
CH_DEV uint32_t cta_begin(const Partition &pt, uint32_t c) {
  return pt.aligned ? (c * pt.rq + min(c, pt.rrem)) * pt.KT : part_begin(c * MK_NW, pt.q, pt.rem);
}
CH_DEV uint32_t cta_begin(const GemvOut &o, uint32_t c) { return cta_begin(o.pt, c); }
// first tile of warp w (0..MK_NW) of CTA c
CH_DEV uint32_t warp_begin(const Partition &pt, uint32_t c, uint32_t w) {
  if (!pt.aligned) return part_begin(c * MK_NW + w, pt.q, pt.rem);
  const uint32_t b = cta_begin(pt, c), T = cta_begin(pt, c + 1) - b;
  return b + part_begin(w, T / MK_NW, T % MK_NW);
}
// warp of CTA c (0..MK_NW-1) whose range holds tile t of that CTA
CH_DEV uint32_t warp_of(const Partition &pt, uint32_t c, uint32_t t) {
  if (!pt.aligned) return part_warp_of(t, pt.q, pt.rem) - c * MK_NW;
  const uint32_t b = cta_begin(pt, c), T = cta_begin(pt, c + 1) - b;
  return part_warp_of(t - b, T / MK_NW, T % MK_NW);
}

// tensor parallel: the same buffer in rank r's exchange arena
template <typename T>
CH_DEV T *on_rank(const MegaArgs &a, T *local, uint32_t r) {
  return reinterpret_cast<T *>(a.arena[r] + (reinterpret_cast<const uint8_t *>(local) - a.arena[a.rank]));
}

// ---------------------------------------------------------------------------
// Straddle list of a GEMV output: entry k = c-1 describes the CTA boundary in front
// of CTA c.  When that boundary is the first one inside a row tile rt, the row
// tile is the sum of the partial slots of CTAs c-1 .. c1: slist[k] = rt and
// soff[k] = the two slot offsets (in floats, into the [grid][2][16] partials)
// when c1 == c (the common case), else kNoStraddle (the general sum walks the
// CTAs).  slist[k] = kNoStraddle for boundaries between row tiles.  One thread
// per entry.
// Entry c-1 (c = 1 .. grid-1) of the list of partition pt; computed once per launch
// for every GEMV kind (straddle_lists), since it depends on the partition alone.
CH_DEV void slist_entry(const Partition &pt, uint32_t c, uint32_t *slist, uint32_t *soff) {
  const uint32_t G = gridDim.x, KT = pt.KT;
  const uint32_t B = cta_begin(pt, c);  // first tile of CTA c
  const uint32_t rt = B / KT;
  uint32_t e = kNoStraddle, off = kNoStraddle;
  const uint32_t b0 = cta_begin(pt, c - 1);
  if (B != rt * KT && b0 <= rt * KT) {
    const uint32_t t_hi = rt * KT + KT - 1;
    if (c + 1 >= G || cta_begin(pt, c + 1) > t_hi)  // exactly CTAs c-1 and c
      off = ((c - 1) * 2 + (b0 < rt * KT ? 1u : 0u)) * 16 | ((c * 2) * 16) << 16;
    e = rt;
  }
  slist[c - 1] = e;
  soff[c - 1] = off;
}
// value of row `row` (0..15) of the straddling row tile of entry k from the staged
// CTA partials P[grid][2][16]: the CTAs' sums in CTA order
CH_DEV float straddle_value(const GemvOut &o, const uint32_t *slist, const uint32_t *soff, const float *P,
                            uint32_t k, uint32_t row) {
  const uint32_t off = soff[k];
  if (off != kNoStraddle) return __fadd_rn(__fadd_rn(0.f, P[(off & 0xFFFFu) + row]), P[(off >> 16) + row]);
  const uint32_t t_lo = slist[k] * o.pt.KT, t_hi = t_lo + o.pt.KT - 1;
  float v = 0.f;
  for (uint32_t cc = k; cc < gridDim.x && cta_begin(o, cc) <= t_hi; cc++) {
    const uint32_t b = cta_begin(o, cc);
    if (b == cta_begin(o, cc + 1)) continue;  // CTA without tiles
    v = __fadd_rn(v, P[(cc * 2 + (b < t_lo ? 1u : 0u)) * 16 + row]);
  }
  return v;
}
// rows q .. q+3 (q % 4 == 0) of straddle entry k: 16-byte loads of the two CTAs'
// partial slots when exactly two CTAs share the row tile
CH_DEV float4 straddle_quad(const GemvOut &o, const uint32_t *slist, const uint32_t *soff, const float *P, uint32_t k,
                            uint32_t q) {
  const uint32_t off = soff[k];
  if (off != kNoStraddle) {
    const float4 x = *reinterpret_cast<const float4 *>(P + (off & 0xFFFFu) + q);
    const float4 y = *reinterpret_cast<const float4 *>(P + (off >> 16) + q);
    return make_float4(__fadd_rn(__fadd_rn(0.f, x.x), y.x), __fadd_rn(__fadd_rn(0.f, x.y), y.y),
                       __fadd_rn(__fadd_rn(0.f, x.z), y.z), __fadd_rn(__fadd_rn(0.f, x.w), y.w));
  }
  return make_float4(straddle_value(o, slist, soff, P, k, q), straddle_value(o, slist, soff, P, k, q + 1),
                     straddle_value(o, slist, soff, P, k, q + 2), straddle_value(o, slist, soff, P, k, q + 3));
}
// Patch the straddling rows of staged (non-act) output rows [r0, r1) (both multiples
// of 4; dst 16-byte aligned), dst[i] = row r0 + i; four rows per thread
CH_DEV void patch_staged(const GemvOut &o, const uint32_t *slist, const uint32_t *soff, const float *P, uint32_t r0,
                         uint32_t r1, float *dst) {
  const uint32_t items = (gridDim.x - 1) * 4;
  for (uint32_t idx = threadIdx.x; idx < items; idx += blockDim.x) {
    const uint32_t k = idx >> 2, rt = slist[k];
    if (rt == kNoStraddle) continue;
    const uint32_t q = (idx & 3u) * 4, r = rt * 16 + q;
    if (r >= r0 && r + 4 <= r1) *reinterpret_cast<float4 *>(dst + (r - r0)) = straddle_quad(o, slist, soff, P, k, q);
  }
}

// Grid barrier on a monotonically increasing arrival counter, in two halves so a
// CTA can do work that does not depend on the other CTAs between its arrival
// and its wait.  The wait is bounded.
// Arrival at the barrier after a phase.  Every CTA releases its writes at GPU
// scope (its stores to other GPUs' memory included) and arrives on this GPU's
// counter; for a cross-rank barrier the last local arrival, which has acquired
// all of them through that counter, releases at system scope with one signal per
// rank -- a single system-scope release per rank and phase.
CH_DEV void grid_arrive(const MegaArgs &a, bool cross, unsigned long long local_target) {
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!cross) {
      asm volatile("fence.acq_rel.gpu;" ::: "memory");
      asm volatile("red.relaxed.gpu.global.add.u64 [%0], 1;" ::"l"(a.arrive) : "memory");
    } else {
      asm volatile("fence.acq_rel.gpu;" ::: "memory");
      unsigned long long old;
      asm volatile("atom.acq_rel.gpu.global.add.u64 %0, [%1], 1;" : "=l"(old) : "l"(a.arrive) : "memory");
      if (old + 1 == local_target)  // this GPU is done: one signal per rank
        for (uint32_t r = 0; r < a.world; r++)
          asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(on_rank(a, a.garrive, r)) : "memory");
    }
  }
}
CH_DEV unsigned long long load_acquire_u64(const unsigned long long *p, bool sys) {
  unsigned long long v;
  if (sys)
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  else
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// `abort` (shared): set once a wait of this launch gave up, or when the launch
// started with a peer timeout already recorded -- later waits then return at
// once, so a lost rank costs one bounded wait, not one per phase.
CH_DEV void grid_wait(const unsigned long long *ctr, bool sys, unsigned long long target, uint32_t *err,
                      volatile uint32_t *abort) {
  if (threadIdx.x == 0 && !*abort) {
    if (load_acquire_u64(ctr, sys) < target) {
      const uint64_t t0 = globaltimer_ns();
      for (;;) {
        if (load_acquire_u64(ctr, sys) >= target) break;
        if (globaltimer_ns() - t0 > 2000000000ull) {
          atomicOr(err, DEV_ERR_PEER_TIMEOUT);
          *abort = 1u;
          break;
        }
      }
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// input pairs: pair p = (32-block b = p/4, t = p%4) holds the 8 values at
// k = 32b + 2t + {0,1, 8,9, 16,17, 24,25} -- exactly one lane quad's share of the
// 32-block in the GEMV tiles' B operand
CH_DEV void ld_pair(const float *src, uint32_t p, float (&v)[8]) {
  const float *q = src + (p >> 2) * 32 + (p & 3u) * 2;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const float2 f = *reinterpret_cast<const float2 *>(q + 8 * i);
    v[2 * i] = f.x, v[2 * i + 1] = f.y;
  }
}
CH_DEV void st_pair(float *dst, uint32_t p, const float (&v)[8]) {
  float *q = dst + (p >> 2) * 32 + (p & 3u) * 2;
#pragma unroll
  for (int i = 0; i < 4; i++) *reinterpret_cast<float2 *>(q + 8 * i) = make_float2(v[2 * i], v[2 * i + 1]);
}
// Input limbs of pair p (values v in ld_pair order) -- the GEMV tiles' B operand
// (core.cuh: limb_item / tile_i8).  A pair's limb words take the bytes of floats
// [8p, 8p+8) of its own 32-block, and the block's 4 pairs run on one aligned lane
// quad, so a staged vector converts in place.  sxs = the block scales (K/32 floats).
CH_DEV void pair_to_limbs(const float (&v)[8], uint32_t p, uint2 *xq, float *sxs) {
  const float e[8] = {v[0], v[2], v[1], v[3], v[4], v[6], v[5], v[7]};
  limb_item(e, p >> 2, p & 3u, xq, sxs);
}

// u32 word of a B-fragment array (f16 hi/lo B fragments of tile_mma: [32-block][t][hi | lo] uint4) that holds
// elements (j, j+1), j even, of the K-vector: hi half (hl = 0) or lo half (hl = 1)
CH_DEV uint32_t frag_word(uint32_t j, uint32_t hl) {
  const uint32_t b = j >> 5, k = j & 31u;
  return ((b * 4 + ((k & 7u) >> 1)) * 2 + hl) * 4 + (k >> 3);
}
// f16 hi/lo split of elements (j, j+1) into a B-fragment array (shared or global)
CH_DEV void store_frag_pair(uint32_t *frag, uint32_t j, float v0, float v1) {
  const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
  const __half l0 = __float2half_rn(__fsub_rn(v0, __half2float(h0)));
  const __half l1 = __float2half_rn(__fsub_rn(v1, __half2float(h1)));
  frag[frag_word(j, 0)] = pack_half2(h0, h1);
  frag[frag_word(j, 1)] = pack_half2(l0, l1);
}

// epochs of the low-latency exchanges of this launch start after this value
__shared__ unsigned long long s_xep;
// set when a wait on another rank gave up: later cross-rank waits of the launch return at once
__shared__ uint32_t s_abort;
// an exchange word: the value in the low half, its epoch in the high half -- written
// and read as one 8-byte access, so a reader that sees the epoch sees the value
CH_DEV void st_x64_sys(unsigned long long *p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
CH_DEV unsigned long long ld_x64_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// one finished output row (local index) of a GEMV: local buffer, or every rank's copy
CH_DEV void out_row(const MegaArgs &a, const GemvOut &o, uint32_t row, float v) {
  if (!o.push) {
    o.direct[row] = v;
    return;
  }
  if (o.push == 2) {  // word [epoch parity][this rank][row] of every rank's exchange array
    const unsigned long long ep = s_xep + o.xidx + 1;
    const unsigned long long w = (ep << 32) | __float_as_uint(v);
    const size_t slot = ((size_t)(ep & 1) * a.world + a.rank) * o.row0 + row;
    for (uint32_t r = 0; r < a.world; r++)
      st_x64_sys(reinterpret_cast<unsigned long long *>(on_rank(a, o.direct, r)) + slot, w);
    return;
  }
  for (uint32_t r = 0; r < a.world; r++) on_rank(a, o.direct, r)[o.row0 + row] = v;
}
// act values (j, j+1) (local index, j even) of a gate|up GEMV as B fragments
CH_DEV void out_act_pair(const MegaArgs &a, const GemvOut &o, uint32_t j, float v0, float v1) {
  uint32_t *f = reinterpret_cast<uint32_t *>(o.direct);
  if (!o.push) {
    store_frag_pair(f, j, v0, v1);
    return;
  }
  for (uint32_t r = 0; r < a.world; r++) store_frag_pair(on_rank(a, f, r), o.row0 + j, v0, v1);
}
// Patch the act values of straddling gate|up row tiles (8 per row tile, act index
// rt*8 + i = gelu(gate row i) * up row i+8) into a staged B-fragment array
CH_DEV void patch_act_frag(const GemvOut &o, const uint32_t *slist, const uint32_t *soff, const float *P, uint32_t K,
                           uint32_t *frag) {
  const uint32_t n = (gridDim.x - 1) * 2;
  for (uint32_t idx = threadIdx.x; idx < n; idx += blockDim.x) {  // act values rt*8 + i .. +3, i = 0 / 4
    const uint32_t k = idx >> 1, rt = slist[k];
    if (rt == kNoStraddle) continue;
    const uint32_t i = (idx & 1u) * 4, j = rt * 8 + i;
    if (j + 4 > K) continue;
    const float4 gv = straddle_quad(o, slist, soff, P, k, i), uv = straddle_quad(o, slist, soff, P, k, i + 8);
    store_frag_pair(frag, j, __fmul_rn(gelu_tanh(gv.x), uv.x), __fmul_rn(gelu_tanh(gv.y), uv.y));
    store_frag_pair(frag, j + 2, __fmul_rn(gelu_tanh(gv.z), uv.z), __fmul_rn(gelu_tanh(gv.w), uv.w));
  }
}
// ld_pair without shared-memory bank conflicts: the pairs of one half-warp cover
// four 32-blocks whose same-offset words share banks, so each thread starts its
// four float2 loads at a different group (rotation by b % 4) and rotates back.
CH_DEV void ld_pair_rot(const float *src, uint32_t p, float (&v)[8]) {
  const float *q = src + (p >> 2) * 32 + (p & 3u) * 2;
  const uint32_t r = (p >> 2) & 3u;
  float2 f[4];
#pragma unroll
  for (int i = 0; i < 4; i++) f[i] = *reinterpret_cast<const float2 *>(q + 8 * ((i + r) & 3u));
  // f[i] holds group (i + r) & 3; group g is f[(g - r) & 3]
  if (r & 1u) {
    const float2 t = f[3];
    f[3] = f[2], f[2] = f[1], f[1] = f[0], f[0] = t;
  }
  if (r & 2u) {
    float2 t = f[0];
    f[0] = f[2], f[2] = t;
    t = f[1];
    f[1] = f[3], f[3] = t;
  }
#pragma unroll
  for (int g = 0; g < 4; g++) v[2 * g] = f[g].x, v[2 * g + 1] = f[g].y;
}

// ---------------------------------------------------------------------------
// Per-warp weight stream over the GEMV phases, driven by lane 0.  The descriptor
// of the phase after the current one is loaded one transition ahead, so moving
// on to the next phase never waits for memory.
struct Stream {
  uint32_t g, ck, nck, tb, te;  // GEMV stream index, next chunk, chunks of this warp's share, its tiles
  const uint8_t *tiles;
  uint4 nxt0, nxt1;             // raw StreamDesc of stream g + 1
};
CH_DEV void load_desc(const MegaArgs &a, uint32_t g, uint4 &d0, uint4 &d1) {
  if (g < a.nstreams) {
    d0 = __ldg(reinterpret_cast<const uint4 *>(a.streams + g));
    d1 = __ldg(reinterpret_cast<const uint4 *>(a.streams + g) + 1);
  } else {
    d0 = d1 = make_uint4(0u, 0u, 0u, 0u);
  }
}
// StreamDesc {tiles, Partition{KT, q, rem, aligned, rq, rrem}} from its two 16-byte halves
CH_DEV void stream_enter(uint32_t gw, Stream &s, const uint4 &d0, const uint4 &d1) {
  s.tiles = reinterpret_cast<const uint8_t *>((uint64_t)d0.x | ((uint64_t)d0.y << 32));
  const Partition pt{d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
  s.tb = warp_begin(pt, gw / MK_NW, gw % MK_NW);
  s.te = warp_begin(pt, gw / MK_NW, gw % MK_NW + 1);
  s.nck = (s.te - s.tb + MK_CT - 1) / MK_CT;
  s.ck = 0;
}
CH_DEV void stream_init(const MegaArgs &a, uint32_t gw, Stream &s) {
  s.g = 0;
  uint4 d0, d1;
  load_desc(a, 0, d0, d1);
  stream_enter(gw, s, d0, d1);
  load_desc(a, 1, s.nxt0, s.nxt1);
}
// advance to the next chunk to issue; false when the step's stream is done
CH_DEV bool stream_next(const MegaArgs &a, uint32_t gw, Stream &s) {
  while (s.ck >= s.nck) {
    if (s.g + 1 >= a.nstreams) return false;
    s.g++;
    stream_enter(gw, s, s.nxt0, s.nxt1);
    load_desc(a, s.g + 1, s.nxt0, s.nxt1);
  }
  return true;
}
CH_DEV void stream_issue(Stream &s, uint8_t *stage, uint64_t *bar, uint64_t pol) {
  const uint32_t t0 = s.tb + s.ck * MK_CT;
  const uint32_t bytes = min((uint32_t)MK_CT, s.te - t0) * kTileBytes;
  mbar_arrive_expect_tx(bar, bytes);
  bulk_g2s_hint(stage, s.tiles + (size_t)t0 * kTileBytes, bytes, bar, pol);
  s.ck++;
}

// phase struct -> shared memory with asynchronous 16-byte copies (threads 0..)
CH_DEV void copy_phase(const Phase *src, Phase *dst) {
  constexpr uint32_t n = sizeof(Phase) / 16;
  static_assert(sizeof(Phase) % 16 == 0, "Phase is copied in 16-byte pieces");
  if (threadIdx.x < n)
    cp_async16(reinterpret_cast<uint8_t *>(dst) + threadIdx.x * 16,
               reinterpret_cast<const uint8_t *>(src) + threadIdx.x * 16);
}

// The row tiles of CTA c that a GEMV of partition pt leaves to the CTA combine (cut
// between warps of the CTA, or straddling a CTA boundary), one item each:
// {rt, w0 | w1 << 4 | inside << 8 | CTA slot << 9 | warp slot bits of w0..w1 << 16}.
// Depends on the partition alone, so it is computed once per launch (comb_items).
CH_DEV bool comb_item(const Partition &pt, uint32_t c, uint32_t rt, uint2 &item) {
  const uint32_t KT = pt.KT, cb = cta_begin(pt, c), ce = cta_begin(pt, c + 1);
  const uint32_t t_lo = rt * KT, t_hi = t_lo + KT - 1;
  const uint32_t a_lo = max(t_lo, cb), a_hi = min(t_hi, ce - 1);
  const uint32_t w0 = warp_of(pt, c, a_lo), w1 = warp_of(pt, c, a_hi);
  const bool inside = cb <= t_lo && t_hi < ce;
  if (w0 == w1 && inside) return false;  // one warp covered the whole row tile: stored by its flush
  uint32_t slots = 0;
  for (uint32_t w = w0; w <= w1; w++)
    if (warp_begin(pt, c, w) < t_lo) slots |= 1u << w;
  item = make_uint2(rt, w0 | w1 << 4 | (inside ? 1u : 0u) << 8 | (cb < t_lo ? 1u : 0u) << 9 | slots << 16);
  return true;
}

// ---------------------------------------------------------------------------
struct SmemLayout {
  uint8_t *stages;
  uint64_t *bars;
  uint64_t *vbar;   // staged activations: two arrivals per phase (before and after the grid barrier)
  uint4 *xzero;     // a zero B fragment (f16 tiles: the lanes without an x column)
  float *wpart;     // [warps][2][16] partial segments of the current GEMV phase
  uint32_t *sl;     // [kKinds][2][g4] straddle lists (entries, partial-slot offsets) of every GEMV kind
  uint32_t g4;      // entries per list: the grid rounded up to a multiple of 4
  uint2 *comb;      // [kKinds][kMaxComb] this CTA's combine items of every GEMV kind
  uint32_t *ncomb;  // [kKinds] their counts
  uint4 *wtab;      // [kKinds][MK_NW] each warp's tile range of every GEMV kind: {first, end, row tile, k tile}
  uint32_t *wphys;  // [2][kWinSlots] attention window slot ids (full, sliding lists)
  uint8_t *u;       // union region (GEMV staging / attention / top-k)
};
// straddle list (and its partial-slot offsets) of the outputs of GEMV kind `kind`
CH_DEV const uint32_t *sl_list(const SmemLayout &L, uint32_t kind) { return L.sl + kind * 2 * L.g4; }
CH_DEV const uint32_t *sl_off(const SmemLayout &L, uint32_t kind) { return L.sl + kind * 2 * L.g4 + L.g4; }
// Once per launch, before the first phase: every kind's straddle list (one thread per
// entry) and this CTA's combine items (one thread per row tile of its range).
CH_DEV void launch_tables(const MegaArgs &a, const SmemLayout &L) {
  const uint32_t G = gridDim.x, c = blockIdx.x;
  if (threadIdx.x < kKinds) L.ncomb[threadIdx.x] = 0u;
  for (uint32_t e = threadIdx.x; e < kKinds * (G - 1); e += blockDim.x) {
    const uint32_t k = e / (G - 1), cc = 1 + e % (G - 1);
    slist_entry(a.kpart[k], cc, L.sl + k * 2 * L.g4, L.sl + k * 2 * L.g4 + L.g4);
  }
  __syncthreads();
  for (uint32_t k = 0; k < kKinds; k++) {
    const Partition &pt = a.kpart[k];
    const uint32_t cb = cta_begin(pt, c), ce = cta_begin(pt, c + 1);
    if (ce == cb) continue;
    const uint32_t rt0 = cb / pt.KT, nrt = (ce - 1) / pt.KT - rt0 + 1;
    for (uint32_t i = threadIdx.x; i < nrt; i += blockDim.x) {
      uint2 item;
      if (!comb_item(pt, c, rt0 + i, item)) continue;
      const uint32_t j = atomicAdd(&L.ncomb[k], 1u);
      if (j < kMaxComb)
        L.comb[k * kMaxComb + j] = item;
      else
        atomicOr(a.err, DEV_ERR_BAD_LIST);  // cannot happen: at most 17 cut row tiles per CTA
    }
  }
  if (threadIdx.x < kKinds * MK_NW) {  // every warp's tile range and its first (row tile, k tile)
    const uint32_t k = threadIdx.x / MK_NW, w = threadIdx.x % MK_NW;
    const Partition &pt = a.kpart[k];
    const uint32_t tb = warp_begin(pt, c, w), te = warp_begin(pt, c, w + 1), rt = tb / pt.KT;
    L.wtab[threadIdx.x] = make_uint4(tb, te, rt, tb - rt * pt.KT);
  }
  __syncthreads();
  if (threadIdx.x < kKinds) L.ncomb[threadIdx.x] = min(L.ncomb[threadIdx.x], kMaxComb);
  __syncthreads();
}
// stage `bytes` from global into shared memory on vbar (any thread)
CH_DEV void stage_copy(const SmemLayout &L, void *dst, const void *src, uint32_t bytes) {
  mbar_expect_tx(L.vbar, bytes);
  bulk_g2s(dst, src, bytes, L.vbar);
}

// GEMV staging in the union region (K floats each): S0 = previous output (norm
// prologues: then its limbs, in place, with their block scales over the start of
// S1; o / down: the producer's B fragments); for the norm prologues S1 = residual,
// S2 = post-norm weight, S3 = norm weight; then the straddle partials of the
// previous GEMV.
CH_DEV uint32_t gemv_stage_vectors(uint32_t pm) { return (pm == PM_NORM || pm == PM_ADD_NORM) ? 4u : 1u; }
struct GemvStage {
  float *s0, *s1, *s2, *s3, *part;
  __device__ GemvStage(uint8_t *u, uint32_t K, uint32_t pm) {
    s0 = reinterpret_cast<float *>(u);
    s1 = s0 + K;
    s2 = s1 + K;
    s3 = s2 + K;
    part = s0 + gemv_stage_vectors(pm) * K;
  }
};

// Sum over the CTA's threads: block_sum's additions in block_sum's order (the warps'
// sums 0 .. MK_NW-1 added to 0), with the MK_NW partials read by four 16-byte loads
// issued together instead of one dependent load per warp.  red: 16-byte aligned.
CH_DEV float cta_sum(float v, float *red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float4 q[MK_NW / 4];
#pragma unroll
  for (int i = 0; i < MK_NW / 4; i++) q[i] = reinterpret_cast<const float4 *>(red)[i];
  float t = 0.0f;
#pragma unroll
  for (int i = 0; i < MK_NW / 4; i++) {
    t += q[i].x;
    t += q[i].y;
    t += q[i].z;
    t += q[i].w;
  }
  return t;
}

// GEMV input.  Norm prologues (q|k|v, gate|up, LM head): the limbs of the normed
// vector, in place over S0, and their block scales over the first K/32 floats after
// it -- integer tiles.  PM_DIRECT / PM_GELU (o, down): S0 already holds the
// producer's f16 hi/lo B fragments (attention out / GELU*up), patched for the
// straddling act values -- f16 tiles; building limbs of those long vectors in every
// CTA (one item per 8 values) cost more than the integer tiles save.
CH_DEV void gemv_prologue(const Phase &p, const MegaArgs &a, const SmemLayout &L, float *red, uint32_t pi) {
  const uint32_t K = p.K, npairs = K / 8, tid = threadIdx.x;
  GemvStage S(L.u, K, p.pm);
  uint2 *xq = reinterpret_cast<uint2 *>(S.s0);
  float *sxs = S.s0 + K;
  const bool writer = (blockIdx.x == 0);
  if (p.pm == PM_DIRECT) return;
  if (p.pm == PM_GELU) {
    patch_act_frag(p.r_in, sl_list(L, p.r_in.kind), sl_off(L, p.r_in.kind), S.part, K,
                   reinterpret_cast<uint32_t *>(S.s0));
    return;
  }
  // PM_NORM / PM_ADD_NORM: one pair per thread (K <= 8 * threads)
  const bool on = tid < npairs;
  float x[8], w[8];
#pragma unroll
  for (int e = 0; e < 8; e++) x[e] = 0.f, w[e] = 0.f;
  if (p.pm == PM_ADD_NORM) {  // x = (x_in + [rmsnorm(r) * post_w]) * scalar     (add_rmsnorm.wgsl:15-51)
    if (on) {  // residual and post-norm weight (staged before the barrier): read while the patch runs
      ld_pair_rot(S.s1, tid, x);
      if (p.post_w) ld_pair_rot(S.s2, tid, w);
    }
    patch_staged(p.r_in, sl_list(L, p.r_in.kind), sl_off(L, p.r_in.kind), S.part, 0, K, S.s0);
    __syncthreads();
    PHASE_MARK(pi, 7);
    float r[8];
#pragma unroll
    for (int e = 0; e < 8; e++) r[e] = 0.f;
    if (on) {
      if (p.nsum > 1) {
        // row-parallel producer: every rank's partial vector, added in rank order (the
        // same sums on every rank), from the exchange words of this step's epoch --
        // polled until they arrive (bounded), no barrier before this phase
        const unsigned long long ep = s_xep + p.r_in.xidx + 1;
        const unsigned long long *q = reinterpret_cast<const unsigned long long *>(p.r_in.direct) +
                                      (size_t)(ep & 1) * p.nsum * K + (tid >> 2) * 32 + (tid & 3u) * 2;
        const uint64_t t0 = globaltimer_ns();
        bool live = !*(volatile uint32_t *)&s_abort;
        // two ranks' 8 words at a time in flight together (one round trip), then checked
        // and added in rank order; a word whose epoch is not here yet is polled alone
        for (uint32_t rk = 0; rk < p.nsum; rk += 2) {
          const uint32_t nr = min(2u, p.nsum - rk);
          unsigned long long w[2][8];
#pragma unroll
          for (uint32_t j = 0; j < 2; j++)
#pragma unroll
            for (int e = 0; e < 8; e++)
              w[j][e] = j < nr ? ld_x64_sys(q + (size_t)(rk + j) * K + 8 * (e >> 1) + (e & 1)) : 0ull;
#pragma unroll
          for (uint32_t j = 0; j < 2; j++) {
            if (j >= nr) break;
#pragma unroll
            for (int e = 0; e < 8; e++) {
              while ((uint32_t)(w[j][e] >> 32) != (uint32_t)ep && live) {
                if (globaltimer_ns() - t0 > 2000000000ull) {
                  atomicOr(a.err, DEV_ERR_PEER_TIMEOUT);
                  s_abort = 1u;
                  live = false;
                }
                w[j][e] = ld_x64_sys(q + (size_t)(rk + j) * K + 8 * (e >> 1) + (e & 1));
              }
              const float v = __uint_as_float((uint32_t)w[j][e]);
              r[e] = (rk + j) ? __fadd_rn(r[e], v) : v;
            }
          }
        }
      } else {
        ld_pair_rot(S.s0, tid, r);
      }
    }
    float inv_r = 1.0f;
    if (p.post_w) {
      float sr = 0.f;
#pragma unroll
      for (int e = 0; e < 8; e++) sr = __fmaf_rn(r[e], r[e], sr);
      sr = cta_sum(sr, red);
      inv_r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sr, (float)K), a.eps)));
    }
#pragma unroll
    for (int e = 0; e < 8; e++) {
      const float rr = p.post_w ? __fmul_rn(__fmul_rn(r[e], inv_r), w[e]) : r[e];
      x[e] = __fmul_rn(__fadd_rn(x[e], rr), p.scalar);
    }
    if (writer && p.x_out && on) st_pair(p.x_out, tid, x);
  } else if (on) {
    ld_pair_rot(S.s1, tid, x);
  }
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 8; e++) ss = __fmaf_rn(x[e], x[e], ss);
  ss = cta_sum(ss, red);  // also orders every read of S0 / S1 before the in-place limb writes
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), a.eps)));
  if (on) {
    float nw[8], v[8];
    ld_pair_rot(S.s3, tid, nw);
#pragma unroll
    for (int e = 0; e < 8; e++) v[e] = __fmul_rn(__fmul_rn(x[e], inv), nw[e]);
    if (writer && p.normed_out) st_pair(p.normed_out, tid, v);
    pair_to_limbs(v, tid, xq, sxs);
  }
}

// After every warp of the CTA finished its tiles: fold the warps' partial segments of
// the row tiles listed for this CTA (comb_item), in warp order.  Row tiles inside the
// CTA's range go to `direct`, straddling ones to the CTA's slot.
CH_DEV void cta_combine(const Phase &p, const MegaArgs &a, const SmemLayout &L) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t c = blockIdx.x, kind = p.out.kind;
  const uint2 *items = L.comb + kind * kMaxComb;
  const uint32_t n = L.ncomb[kind];
  for (uint32_t j = warp; j < n; j += MK_NW) {
    const uint2 it = items[j];
    const uint32_t rt = it.x, w0 = it.y & 15u, w1 = (it.y >> 4) & 15u;
    const bool inside = (it.y >> 8) & 1u;
    // every warp's segment loaded first (all in range of wpart), then added in warp order
    float seg[MK_NW];
#pragma unroll
    for (int w = 0; w < MK_NW; w++) seg[w] = L.wpart[(w * 2 + ((it.y >> (16 + w)) & 1u)) * 16 + (lane & 15)];
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < MK_NW; w++)
      if ((uint32_t)w >= w0 && (uint32_t)w <= w1) sum = __fadd_rn(sum, seg[w]);
    if (lane >= 16) sum = 0.f;
    const float up = __shfl_down_sync(0xffffffffu, sum, 8);
    if (inside) {
      if (p.out.act) {  // act values of lanes 0..7 as B fragments, in pairs
        const float av = __fmul_rn(gelu_tanh(sum), up);
        const float an = __shfl_down_sync(0xffffffffu, av, 1);
        if (lane < 8 && !(lane & 1)) out_act_pair(a, p.out, rt * 8 + lane, av, an);
      } else if (lane < 16) {
        out_row(a, p.out, rt * 16 + lane, sum);
      }
    } else if (lane < 16) {  // straddling row tile: this CTA's share, added up by the consumer
      p.out.partial[((size_t)c * 2 + ((it.y >> 9) & 1u)) * 16 + lane] = sum;
    }
  }
}

// LIMBS: integer tiles against the input limbs (xq, sxs); else f16 tiles against the
// f16 hi/lo B fragments at xq (sxs unused)
template <int FMT, bool LIMBS>
CH_DEV void gemv_tiles(const Phase &p, const MegaArgs &a, uint32_t gw, const SmemLayout &L, const uint2 *xq,
                       const float *sxs, uint32_t &cidx, Stream &st, bool &ok, uint64_t pol, uint32_t pi) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  uint8_t *my_stages = L.stages + (size_t)warp * MK_SPW * MK_STAGE;
  uint64_t *my_bars = L.bars + warp * MK_SPW;
  const uint32_t KT = p.k_tiles;
  const uint4 wt = L.wtab[p.out.kind * MK_NW + warp];  // {first tile, end, its row tile, its k tile}
  const uint32_t tb = wt.x, te = wt.y;
  const uint32_t nchunks = (te - tb + MK_CT - 1) / MK_CT;
  const uint2 *xql = xq + t * 4 + (g & 3);
  // f16 path: lanes g < 2 read the hi / lo column, the others a zero page
  const uint4 *xb = (g < 2) ? reinterpret_cast<const uint4 *>(xq) + t * 2 + g : L.xzero;
  const uint32_t xs = (g < 2) ? 8u : 0u;
  uint32_t rt = wt.z, kt = wt.w, cur_rt = 0xFFFFFFFFu, kt_begin = 0;
  float acc[4] = {0.f, 0.f, 0.f, 0.f}, accb[4] = {0.f, 0.f, 0.f, 0.f};  // two chains (even / odd tiles)
  bool first_seg = true;
  auto tile = [&](const uint8_t *tp, uint32_t k, float(&ac)[4]) {
    if constexpr (LIMBS)
      tile_i8<FMT>(tp, k, xql, sxs, lane, ac);
    else
      tile_mma<FMT>(tp, k, xb, xs, lane, ac[0], ac[1]);
  };
  auto flush = [&](uint32_t frt, uint32_t kb, uint32_t ke) {
    float acc0, acc1;
    if constexpr (LIMBS) {
      limb_rows<FMT>(acc, accb, t, acc0, acc1);
    } else {
      acc0 = __fadd_rn(acc[0], accb[0]);
      acc1 = __fadd_rn(acc[1], accb[1]);
    }
    // act mode: lanes t == 0 hold act value g of the row tile; pair g, g+1 (lane + 4)
    const float av = __fmul_rn(gelu_tanh(acc0), acc1);
    const float an = __shfl_down_sync(0xffffffffu, av, 4);
    if (t == 0) {
      if (kb == 0 && ke == KT) {
        if (p.out.act) {
          if (!(g & 1)) out_act_pair(a, p.out, frt * 8 + g, av, an);
        } else {
          out_row(a, p.out, frt * 16 + g, acc0);
          out_row(a, p.out, frt * 16 + g + 8, acc1);
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
    if (j == 0) {
      WARP_MARK(pi, 8, 0);
      WARP_MARK(pi, 10, MK_NW - 1);
    }
    const uint8_t *stg = my_stages + (size_t)s * MK_STAGE;
    const uint32_t t0 = tb + j * MK_CT;
    const uint32_t nt = min((uint32_t)MK_CT, te - t0);
    uint32_t i = 0;
    while (i < nt) {
      if (rt != cur_rt) {
        if (cur_rt != 0xFFFFFFFFu) flush(cur_rt, kt_begin, KT);
        cur_rt = rt;
        kt_begin = kt;
#pragma unroll
        for (int c = 0; c < 4; c++) acc[c] = accb[c] = 0.f;
      }
      const uint32_t run = min(nt - i, KT - kt);
      const uint8_t *pp = stg + (size_t)i * kTileBytes;
      uint32_t r = 0;
      if (run == MK_CT) {
#pragma unroll
        for (int q = 0; q + 1 < MK_CT; q += 2) {
          tile(pp + q * kTileBytes, kt + q, acc);
          tile(pp + (q + 1) * kTileBytes, kt + q + 1, accb);
        }
        if constexpr (MK_CT % 2) tile(pp + (MK_CT - 1) * kTileBytes, kt + MK_CT - 1, acc);
        r = MK_CT;
      } else {
        for (; r + 2 <= run; r += 2) {
          tile(pp + r * kTileBytes, kt + r, acc);
          tile(pp + (r + 1) * kTileBytes, kt + r + 1, accb);
        }
        if (r < run) tile(pp + r * kTileBytes, kt + r, acc);
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
      stream_issue(st, my_stages + (size_t)s * MK_STAGE, &my_bars[s], pol);
    }
    __syncwarp();
  }
  if (cur_rt != 0xFFFFFFFFu) flush(cur_rt, kt_begin, te - cur_rt * KT);
  WARP_MARK(pi, 9, 0);
  WARP_MARK(pi, 11, MK_NW - 1);
}

// ---------------------------------------------------------------------------
// ATTN phase: work item (kv head, slot chunk) per CTA; qkv_rope.wgsl + decode_attn.wgsl
struct AttnItem {
  uint32_t S, nsplit, chunk, kvh, split, c0, n;
  const uint32_t *list;
  bool active;
};
CH_DEV AttnItem attn_item(const MegaArgs &a, const StepParams &sp, uint32_t is_sliding) {
  AttnItem it;
  it.S = is_sliding ? sp.n_sliding : sp.n_active;
  it.list = is_sliding ? sp.sliding : sp.active;
  it.chunk = max(kMinChunk, (it.S + a.attn_max_splits - 1) / a.attn_max_splits);
  it.nsplit = it.S == 0 ? 1u : (it.S + it.chunk - 1) / it.chunk;
  const uint32_t item = blockIdx.x;
  it.active = item < a.nkv * it.nsplit;
  it.kvh = item / it.nsplit;
  it.split = item % it.nsplit;
  it.c0 = it.split * it.chunk;
  const uint32_t c1 = min(it.S, it.c0 + it.chunk);
  it.n = c1 > it.c0 ? c1 - it.c0 : 0;
  return it;
}

// attention output elements (j, j+1) of this rank's heads as B fragments of the
// o-projection input: local buffer (one GPU, or tensor parallel with a row-parallel o
// projection reading this rank's heads only), or every rank's copy at the rank's
// global head offset
CH_DEV void attn_out_pair(const MegaArgs &a, uint32_t *frag, uint32_t j, float v0, float v1) {
  if (a.world <= 1 || a.attn_local) {
    store_frag_pair(frag, j, v0, v1);
    return;
  }
  for (uint32_t r = 0; r < a.world; r++) store_frag_pair(on_rank(a, frag, r), a.attn_q0 * kHeadDim + j, v0, v1);
}

// Shared-memory layout of the ATTN phase (inside the union region).
template <int R>
struct AttnSmem {
  static constexpr int D = kHeadDim;
  float *q_s;      // [R][D] q heads (staged raw, normed + roped in place)
  float *k_new;    // [D]   this step's K row (staged raw, then f16-rounded)
  float *v_new;    // [D]
  float *qn_w;     // [D]   q_norm weight      (staged before the barrier)
  float *kn_w;     // [D]   k_norm weight      (staged before the barrier)
  float2 *cs;      // [D/2] RoPE (cos, sin)    (staged before the barrier)
  __half *kv;      // [2][kWinSlots][D] K then V rows of the window (staged before the barrier)
  float *o_s;      // [MK_NW][R][D] per-warp P*V (overlays kv once scores and P*V are done)
  float *sc;       // [R][chunk_cap]
  float *cmb;      // [R][max_splits] split maxima, then weights
  float *cml;      // [R][max_splits] split sums
  float *stat;     // [2R]
  float *part;     // [grid][2][16] straddle partials of the q|k|v GEMV
  __device__ AttnSmem(uint8_t *u, uint32_t chunk_cap, uint32_t max_splits) {
    q_s = reinterpret_cast<float *>(u);
    k_new = q_s + R * D;
    v_new = k_new + D;
    qn_w = v_new + D;
    kn_w = qn_w + D;
    cs = reinterpret_cast<float2 *>(kn_w + D);
    kv = reinterpret_cast<__half *>(cs + D / 2);
    o_s = reinterpret_cast<float *>(kv);
    const size_t kv_bytes = (size_t)2 * kWinSlots * D * 2, os_bytes = (size_t)MK_NW * R * D * 4;
    sc = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(kv) + (kv_bytes > os_bytes ? kv_bytes : os_bytes));
    cmb = sc + R * chunk_cap;
    cml = cmb + R * max_splits;
    stat = cml + R * max_splits;
    part = reinterpret_cast<float *>((reinterpret_cast<uintptr_t>(stat + 2 * R) + 15) & ~(uintptr_t)15);
  }
};
CH_DEV uint32_t attn_chunk_cap(const MegaArgs &a) {
  return max(kMinChunk, (a.cache_slots + a.attn_max_splits - 1) / a.attn_max_splits);
}

// Once per step: the window's slot ids of this CTA's work item for the full and the
// sliding lists (the lists do not change within a step).
// The CTA's two work items (full, sliding list) of the step, computed once per launch
// (attn_lists_init) and read by every attention phase.
__shared__ AttnItem s_attn_items[2];
CH_DEV const AttnItem &attn_item_of(uint32_t is_sliding) { return s_attn_items[is_sliding ? 1 : 0]; }

CH_DEV void attn_lists_init(const MegaArgs &a, const StepParams &sp, uint32_t *wphys) {
  if (threadIdx.x < 2) s_attn_items[threadIdx.x] = attn_item(a, sp, threadIdx.x);
  for (uint32_t v = 0; v < 2; v++) {
    const AttnItem it = attn_item(a, sp, v);
    for (uint32_t i = threadIdx.x; i < kWinSlots; i += MK_THREADS)
      wphys[v * kWinSlots + i] = (it.active && i < it.n) ? __ldcg(it.list + it.c0 + i) : 0xFFFFFFFFu;
  }
}

// before the barrier: the window's K/V rows as 16-byte cp.async pieces (each thread
// waits for its own in attn_phase; one bulk copy per 512-byte row measured slower),
// bulk copies of the head norm weights and the RoPE table, and the chunk's slots
// beyond the window toward L2
template <int R>
CH_DEV void attn_pre(const Phase &p, const MegaArgs &a, const StepParams &sp, const SmemLayout &L) {
  constexpr int D = kHeadDim;
  const AttnItem &it = attn_item_of(p.is_sliding);
  if (!it.active) return;
  AttnSmem<R> sm(L.u, attn_chunk_cap(a), a.attn_max_splits);
  const size_t kv_dim = (size_t)a.nkv * D;
  const uint32_t *wp = L.wphys + p.is_sliding * kWinSlots;
  const uint32_t t = threadIdx.x;
  if (t == 0) {
    stage_copy(L, sm.qn_w, p.q_norm_w, D * 4);
    stage_copy(L, sm.kn_w, p.k_norm_w, D * 4);
    stage_copy(L, sm.cs, p.rope_cs, a.rot * 4);  // rot/2 (cos, sin) pairs
  }
  constexpr uint32_t kPieces = D * 2 / 16;  // 16-byte pieces per row
  for (uint32_t piece = t; piece < 2 * kWinSlots * kPieces; piece += MK_THREADS) {
    const uint32_t row = piece / kPieces, sub = piece % kPieces;
    const uint32_t which = row / kWinSlots, i = row % kWinSlots;  // K rows, then V rows
    if (i >= it.n) continue;
    const uint32_t phys = wp[i];
    if (phys >= a.cache_slots || phys == sp.slot) continue;
    cp_async16(sm.kv + (size_t)row * D + sub * 8,
               (which ? p.v_cache : p.k_cache) + (size_t)phys * kv_dim + (size_t)it.kvh * D + sub * 8);
  }
  for (uint32_t i = kWinSlots + threadIdx.x; i < it.n; i += MK_THREADS) {
    const uint32_t phys = __ldcg(it.list + it.c0 + i);
    if (phys < a.cache_slots) {
      const size_t off = (size_t)phys * kv_dim + (size_t)it.kvh * D;
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p.k_cache + off));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p.k_cache + off + 128));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p.v_cache + off));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p.v_cache + off + 128));
    }
  }
}
// right after the barrier (thread 0): this kv head's q | k | v rows and the q|k|v partials
template <int R>
CH_DEV void attn_post_copies(const Phase &p, const MegaArgs &a, const StepParams &sp, const SmemLayout &L) {
  constexpr int D = kHeadDim;
  const AttnItem &it = attn_item_of(p.is_sliding);
  if (!it.active) return;
  AttnSmem<R> sm(L.u, attn_chunk_cap(a), a.attn_max_splits);
  const uint32_t kvh = it.kvh, kv_dim = a.nkv * D;
  stage_copy(L, sm.q_s, p.r_in.direct + kvh * R * D, R * D * 4);
  stage_copy(L, sm.k_new, p.r_in.direct + a.nq * D + kvh * D, D * 4);
  stage_copy(L, sm.v_new, p.r_in.direct + a.nq * D + kv_dim + kvh * D, D * 4);
  stage_copy(L, sm.part, p.r_in.partial, gridDim.x * 32 * 4);
}

template <int R>
CH_DEV void attn_phase(const Phase &p, const MegaArgs &a, const StepParams &sp, const SmemLayout &L, uint32_t pi) {
  constexpr int D = kHeadDim, EPL = 8;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const AttnItem &it = attn_item_of(p.is_sliding);
  if (!it.active) return;
  const uint32_t max_splits = a.attn_max_splits, n = it.n, kvh = it.kvh;
  const size_t kv_dim = (size_t)a.nkv * D;
  const uint32_t chunk_cap = attn_chunk_cap(a);
  AttnSmem<R> sm(L.u, chunk_cap, max_splits);
  const uint32_t *wp = L.wphys + p.is_sliding * kWinSlots;

  // 0. straddling rows of the staged heads (q heads, k, v: three row ranges, each a
  //    multiple of 4 rows, so a quad of rows never crosses one)
  {
    const uint32_t n4 = (gridDim.x - 1) * 4;
    const uint32_t q0 = kvh * R * D, k0 = a.nq * D + kvh * D, v0 = a.nq * D + (uint32_t)kv_dim + kvh * D;
    for (uint32_t idx = tid; idx < n4; idx += MK_THREADS) {
      const uint32_t e = sl_list(L, p.r_in.kind)[idx / 4];
      if (e == kNoStraddle) continue;
      const uint32_t q = (idx % 4) * 4, r = (e & 0xFFFFu) * 16 + q;
      float *dst = nullptr;
      if (r >= q0 && r < q0 + R * D) dst = sm.q_s + (r - q0);
      else if (r >= k0 && r < k0 + D) dst = sm.k_new + (r - k0);
      else if (r >= v0 && r < v0 + D) dst = sm.v_new + (r - v0);
      if (dst)
        *reinterpret_cast<float4 *>(dst) =
            straddle_quad(p.r_in, sl_list(L, p.r_in.kind), sl_off(L, p.r_in.kind), sm.part, idx / 4, q);
    }
  }
  __syncthreads();
  PHASE_MARK(pi, 7);
  // 1. q heads | k | v of this kv head: warp h norms and ropes head h in registers, in place
  if (warp < R + 2) {
    float *hd = warp < R ? sm.q_s + warp * D : (warp == R ? sm.k_new : sm.v_new);
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; e++) v[e] = hd[lane * 8 + e];
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; e++) ss = __fmaf_rn(v[e], v[e], ss);
    ss = warp_sum(ss);
    // ss / D as ss * 2^-8: D = 256 is a power of two, so both round the same exact value
    static_assert(D == 256, "the head mean below divides by 256");
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(ss, 1.0f / 256.0f), a.eps)));
    float out[8];
    if (warp <= R) {  // rmsnorm * w, then RoPE half-split at `clock` (qkv_rope.wgsl; kernels.zig:101-119)
      const float *w = warp < R ? sm.qn_w : sm.kn_w;
      float y[8], part[8];
#pragma unroll
      for (int e = 0; e < 8; e++) y[e] = __fmul_rn(__fmul_rn(v[e], inv), w[lane * 8 + e]);
      const uint32_t half = a.rot / 2, lh = half / 8;
      const int src = (uint32_t)lane < lh ? lane + (int)lh : lane - (int)lh;
#pragma unroll
      for (int e = 0; e < 8; e++) part[e] = __shfl_sync(0xffffffffu, y[e], src);
#pragma unroll
      for (int e = 0; e < 8; e++) {
        const uint32_t d = lane * 8 + e;
        if (d < half) {
          const float2 c = sm.cs[d];
          out[e] = __fsub_rn(__fmul_rn(y[e], c.x), __fmul_rn(part[e], c.y));
        } else if (d < a.rot) {
          const float2 c = sm.cs[d - half];
          out[e] = __fadd_rn(__fmul_rn(part[e], c.y), __fmul_rn(y[e], c.x));
        } else {
          out[e] = y[e];
        }
      }
    } else {  // v: unit rmsnorm
#pragma unroll
      for (int e = 0; e < 8; e++) out[e] = __fmul_rn(v[e], inv);
    }
    if (warp >= R) {  // f16 cache row of the new K / V (written by split 0); scores use the rounded values
      __half hv[8];
#pragma unroll
      for (int e = 0; e < 8; e++) {
        hv[e] = __float2half_rn(out[e]);
        out[e] = __half2float(hv[e]);
      }
      if (it.split == 0 && sp.slot < a.cache_slots) {
        __half *dst = (warp == R ? p.k_cache : p.v_cache) + (size_t)sp.slot * kv_dim + (size_t)kvh * D + lane * 8;
        *reinterpret_cast<uint4 *>(dst) = make_uint4(pack_half2(hv[0], hv[1]), pack_half2(hv[2], hv[3]),
                                                     pack_half2(hv[4], hv[5]), pack_half2(hv[6], hv[7]));
      }
    }
    __syncwarp();
    *reinterpret_cast<float4 *>(hd + lane * 8) = make_float4(out[0], out[1], out[2], out[3]);
    *reinterpret_cast<float4 *>(hd + lane * 8 + 4) = make_float4(out[4], out[5], out[6], out[7]);
  }
  if (it.split == 0 && sp.slot >= a.cache_slots && tid == 0) atomicOr(a.err, DEV_ERR_BAD_SLOT);
  cp_async_wait_all();  // this thread's pieces of the K/V window (attn_pre)
  __syncthreads();
  PHASE_MARK(pi, 2);

  // 2. scores: warp w takes slots w, w+16, ...; lane holds d = lane*8 .. +7
  float qr[R][EPL];
#pragma unroll
  for (int h = 0; h < R; h++)
#pragma unroll
    for (int e = 0; e < EPL; e++) qr[h][e] = sm.q_s[h * D + lane * EPL + e];
  auto unpack = [&](const uint4 &rw, float (&f)[EPL]) {
    const __half2 *hp = reinterpret_cast<const __half2 *>(&rw);
#pragma unroll
    for (int e = 0; e < EPL / 2; e++) {
      const float2 x = __half22float2(hp[e]);
      f[2 * e] = x.x;
      f[2 * e + 1] = x.y;
    }
  };
  // row of slot i (window slots from shared memory, the rest from global / L2)
  auto row = [&](uint32_t i, uint32_t which, float (&f)[EPL], uint32_t &phys) {
    phys = i < kWinSlots ? wp[i] : __ldcg(it.list + it.c0 + i);
    if (phys == sp.slot) {
      const float *src = which ? sm.v_new : sm.k_new;
#pragma unroll
      for (int e = 0; e < EPL; e++) f[e] = src[lane * EPL + e];
    } else if (phys < a.cache_slots) {
      if (i < kWinSlots)
        unpack(*reinterpret_cast<const uint4 *>(sm.kv + (size_t)(which * kWinSlots + i) * D + lane * EPL), f);
      else
        unpack(__ldcg(reinterpret_cast<const uint4 *>((which ? p.v_cache : p.k_cache) + (size_t)phys * kv_dim +
                                                       (size_t)kvh * D + lane * EPL)),
               f);
    } else {
#pragma unroll
      for (int e = 0; e < EPL; e++) f[e] = 0.f;
    }
  };
  // two slots (i, i + MK_NW) per iteration: independent chains, each slot's arithmetic unchanged
  for (uint32_t i = warp; i < n; i += 2 * MK_NW) {
    const uint32_t i2 = i + MK_NW;
    const bool two = i2 < n;
    float kv[EPL], kv2[EPL];
    uint32_t phys, phys2 = 0u;
    row(i, 0, kv, phys);
    if (two) {
      row(i2, 0, kv2, phys2);
    } else {
#pragma unroll
      for (int e = 0; e < EPL; e++) kv2[e] = 0.f;
    }
    const bool valid = phys < a.cache_slots, valid2 = phys2 < a.cache_slots;
#pragma unroll
    for (int h = 0; h < R; h++) {
      float dot = 0.f, dot2 = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; e++) {
        dot = __fmaf_rn(qr[h][e], kv[e], dot);
        dot2 = __fmaf_rn(qr[h][e], kv2[e], dot2);
      }
      dot = warp_sum(dot);
      dot2 = warp_sum(dot2);
      if (lane == 0) {
        sm.sc[h * chunk_cap + i] = valid ? __fmul_rn(dot, p.attn_scale) : -INFINITY;
        if (two) sm.sc[h * chunk_cap + i2] = valid2 ? __fmul_rn(dot2, p.attn_scale) : -INFINITY;
      }
    }
    if (lane == 0 && (!valid || (two && !valid2))) atomicOr(a.err, DEV_ERR_BAD_LIST);
  }
  __syncthreads();
  // 3. softmax statistics per head over this chunk (max seeded at -1e9, decode_attn.wgsl:81)
  for (int h = warp; h < R; h += MK_NW) {
    float m = -1e9f;
    for (uint32_t i = lane; i < n; i += 32) m = fmaxf(m, sm.sc[h * chunk_cap + i]);
    m = warp_max(m);
    float l = 0.f;
    for (uint32_t i = lane; i < n; i += 32) {
      const float e = expf(__fsub_rn(sm.sc[h * chunk_cap + i], m));
      sm.sc[h * chunk_cap + i] = e;
      l = __fadd_rn(l, e);
    }
    l = warp_sum(l);
    if (lane == 0) {
      sm.stat[2 * h] = m;
      sm.stat[2 * h + 1] = l;
    }
  }
  __syncthreads();
  // 4. weighted V: every warp over its slots, then a fixed-order sum over warps
  {
    float acc[R][EPL];
#pragma unroll
    for (int h = 0; h < R; h++)
#pragma unroll
      for (int e = 0; e < EPL; e++) acc[h][e] = 0.f;
    for (uint32_t i = warp; i < n; i += MK_NW) {
      float vv[EPL];
      uint32_t phys;
      row(i, 1, vv, phys);
#pragma unroll
      for (int h = 0; h < R; h++) {
        const float pr_ = sm.sc[h * chunk_cap + i];
#pragma unroll
        for (int e = 0; e < EPL; e++) acc[h][e] = __fmaf_rn(pr_, vv[e], acc[h][e]);
      }
    }
    __syncthreads();  // o_s overlays the K/V window
#pragma unroll
    for (int h = 0; h < R; h++) {
      float *dst = sm.o_s + (warp * R + h) * D + lane * EPL;
      *reinterpret_cast<float4 *>(dst) = make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
      *reinterpret_cast<float4 *>(dst + 4) = make_float4(acc[h][4], acc[h][5], acc[h][6], acc[h][7]);
    }
  }
  __syncthreads();
  uint32_t *attn_o = reinterpret_cast<uint32_t *>(p.attn_out);  // B fragments of the o-projection input
  if (it.nsplit == 1) {  // whole list in this CTA: normalize and write (same arithmetic as a 1-split combine)
    for (int idx = tid; idx < R * D; idx += MK_THREADS) {  // R*D is a multiple of 32: whole warps
      const int h = idx / D, d = idx % D;
      float ow[MK_NW];
#pragma unroll
      for (int w = 0; w < MK_NW; w++) ow[w] = sm.o_s[(w * R + h) * D + d];
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < MK_NW; w++) s = __fadd_rn(s, ow[w]);
      const float Lsum = __fmaf_rn(sm.stat[2 * h + 1], 1.0f, 0.f);
      const float o = __fmul_rn(__fmaf_rn(s, 1.0f, 0.f), __fdiv_rn(1.0f, __fadd_rn(Lsum, 1e-9f)));
      const float on = __shfl_down_sync(0xffffffffu, o, 1);
      if (!(idx & 1)) attn_out_pair(a, attn_o, (kvh * R + h) * D + d, o, on);
    }
    return;
  }
  float *part = a.attn_partial + ((size_t)(kvh * max_splits + it.split) * R) * (D + 2);
  for (int idx = tid; idx < R * D; idx += MK_THREADS) {
    const int h = idx / D, d = idx % D;
    float ow[MK_NW];
#pragma unroll
    for (int w = 0; w < MK_NW; w++) ow[w] = sm.o_s[(w * R + h) * D + d];
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < MK_NW; w++) s = __fadd_rn(s, ow[w]);
    part[h * (D + 2) + d] = s;
  }
  if (tid < R) {
    part[tid * (D + 2) + D] = sm.stat[2 * tid];
    part[tid * (D + 2) + D + 1] = sm.stat[2 * tid + 1];
  }
  PHASE_MARK(pi, 3);
  // 5. publish, wait for every split of this kv head (all CTAs of the cooperative grid
  //    are resident), then each split combines its own slice of the R*D outputs
  __threadfence();
  __syncthreads();
  const uint32_t nsplit = it.nsplit;
  if (tid == 0) {
    atomicAdd(&a.attn_counters[kvh], 1u);
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(&a.attn_counters[kvh]) : "memory");
    if (v < nsplit && !(*(volatile uint32_t *)a.err & DEV_ERR_PEER_TIMEOUT)) {
      const uint64_t t0 = globaltimer_ns();
      for (;;) {
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(&a.attn_counters[kvh]) : "memory");
        if (v >= nsplit) break;
        if (globaltimer_ns() - t0 > 2000000000ull) {
          atomicOr(a.err, DEV_ERR_PEER_TIMEOUT);
          break;
        }
      }
    }
  }
  __syncthreads();
  const float *base = a.attn_partial + ((size_t)kvh * max_splits * R) * (D + 2);
  const uint32_t per = (((R * D + nsplit - 1) / nsplit) + 1) & ~1u, i0 = it.split * per;  // even: whole pairs
  const uint32_t i1 = min(i0 + per, (uint32_t)(R * D));
  const uint32_t idx = i0 + tid;
  const bool mine = idx < i1;
  const int h = (int)(idx / D), d = (int)(idx % D);
  float pv[kMkMaxSplits];
#pragma unroll
  for (uint32_t j = 0; j < kMkMaxSplits; j++)
    pv[j] = (j < nsplit && mine) ? __ldcg(&base[((size_t)j * R + h) * (D + 2) + d]) : 0.f;
  for (int s2 = tid; s2 < R * (int)nsplit; s2 += MK_THREADS) {
    const int hh = s2 / nsplit, j = s2 % nsplit;
    const float2 ml = __ldcg(reinterpret_cast<const float2 *>(&base[((size_t)j * R + hh) * (D + 2) + D]));
    sm.cmb[hh * max_splits + j] = ml.x;
    sm.cml[hh * max_splits + j] = ml.y;
  }
  __syncthreads();
  if (warp < R) {  // warp h: lane j holds split j's maximum; the factors in parallel, the sum in split order
    const int hh = warp;
    const float mj = (uint32_t)lane < nsplit ? sm.cmb[hh * max_splits + lane] : -INFINITY;
    const float M = warp_max(mj);
    const float f = (uint32_t)lane < nsplit ? expf(__fsub_rn(mj, M)) : 0.f;
    const float lj = (uint32_t)lane < nsplit ? sm.cml[hh * max_splits + lane] : 0.f;
    float Lsum = 0.f;
#pragma unroll
    for (uint32_t j = 0; j < kMkMaxSplits; j++) {
      const float fj = __shfl_sync(0xffffffffu, f, j), lsj = __shfl_sync(0xffffffffu, lj, j);
      if (j < nsplit) Lsum = __fmaf_rn(lsj, fj, Lsum);
    }
    __syncwarp();
    if ((uint32_t)lane < nsplit) sm.cmb[hh * max_splits + lane] = f;
    if (lane == 0) sm.stat[2 * hh] = __fdiv_rn(1.0f, __fadd_rn(Lsum, 1e-9f));
  }
  __syncthreads();
  float o = 0.f;
  if (mine) {
    float O = 0.f;
#pragma unroll
    for (uint32_t j = 0; j < kMkMaxSplits; j++)
      if (j < nsplit) O = __fmaf_rn(pv[j], sm.cmb[h * max_splits + j], O);
    o = __fmul_rn(O, sm.stat[2 * h]);
  }
  const float on = __shfl_down_sync(0xffffffffu, o, 1);
  if (mine && !(idx & 1)) attn_out_pair(a, attn_o, (kvh * R + h) * D + d, o, on);
}

// ---------------------------------------------------------------------------
// TOPK phase: each CTA selects the top 64 of its vocab slice, last CTA merges
struct TopkSmem {
  uint32_t *hist, *sh, *cnt;
  uint64_t *buf, *sorted;
  float *lg;    // staged logits [lo4, hi4) of this CTA's slice (4-aligned)
  float *part;  // [grid][2][16] straddle partials of the LM head
  __device__ TopkSmem(uint8_t *u) {
    hist = reinterpret_cast<uint32_t *>(u);
    sh = hist + 256;
    cnt = sh + 4;
    buf = reinterpret_cast<uint64_t *>(cnt + 4);
    sorted = buf + 64;
    lg = reinterpret_cast<float *>(sorted + 64);
    part = lg + 4096 + 8;
  }
};
CH_DEV void topk_slice(const Phase &p, uint32_t &lo, uint32_t &hi) {
  const uint32_t G = gridDim.x, V = p.vocab;
  lo = (uint32_t)(((uint64_t)V * blockIdx.x) / G);
  hi = (uint32_t)(((uint64_t)V * (blockIdx.x + 1)) / G);
}
CH_DEV void topk_post_copies(const Phase &p, const SmemLayout &L) {
  TopkSmem sm(L.u);
  uint32_t lo, hi;
  topk_slice(p, lo, hi);
  const uint32_t lo4 = lo & ~3u, hi4 = (hi + 3u) & ~3u;
  if (hi4 > lo4) stage_copy(L, sm.lg, p.r_in.direct + lo4, (hi4 - lo4) * 4);
  stage_copy(L, sm.part, p.r_in.partial, gridDim.x * 32 * 4);
}
// the final 64 (sorted keys) -> ids / vals / greedy token / device-loop step
CH_DEV void topk_finish(const MegaArgs &a, const uint64_t *sorted) {
  const int tid = threadIdx.x;
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
      }
    }
  }
}
CH_DEV void topk_phase(const Phase &p, const MegaArgs &a, const SmemLayout &L) {
  constexpr int E1 = 8, E2 = 20;  // per-thread keys: slice <= 4096, candidates <= 10240
  TopkSmem sm(L.u);
  __shared__ uint32_t last_flag;
  const int tid = threadIdx.x;
  const uint32_t G = gridDim.x;
  uint32_t lo, hi;
  topk_slice(p, lo, hi);
  const uint32_t lo4 = lo & ~3u;
  patch_staged(p.r_in, sl_list(L, p.r_in.kind), sl_off(L, p.r_in.kind), sm.part, lo4, (hi + 3u) & ~3u, sm.lg);
  __syncthreads();
  {
    uint64_t k[E1];
#pragma unroll
    for (int e = 0; e < E1; e++) {
      const uint32_t idx = lo + e * MK_THREADS + tid;
      if (idx < hi) {
        const float v = softcap(sm.lg[idx - lo4]);
        k[e] = ((uint64_t)sortable(v) << 32) | (uint64_t)(0xFFFFFFFFu - (p.vocab0 + idx));  // global id
      } else {
        k[e] = 0;
      }
    }
    const uint64_t thr = block_kth_largest<E1>(k, 64, sm.hist, sm.sh);
    collect_sorted64<E1>(k, thr, sm.buf, sm.cnt, sm.sorted);
    if (tid < 64) a.topk_cand[(size_t)blockIdx.x * 64 + tid] = sm.sorted[tid];
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
  const uint64_t thr = block_kth_largest<E2>(k, 64, sm.hist, sm.sh);
  collect_sorted64<E2>(k, thr, sm.buf, sm.cnt, sm.sorted);
  if (tid == 0) *a.topk_counter = 0u;
  if (a.world <= 1) {
    topk_finish(a, sm.sorted);
    return;
  }
  // tensor parallel: this rank's 64 go to slot `rank` of every rank's candidate table
  if (tid < 64)
    for (uint32_t r = 0; r < a.world; r++) on_rank(a, a.xcand, r)[a.rank * 64 + tid] = sm.sorted[tid];
}

// MERGE phase (tensor parallel): every rank's CTA 0 merges the world x 64 staged
// candidates into the same final 64 and token
CH_DEV void merge_phase(const MegaArgs &a, const SmemLayout &L) {
  if (blockIdx.x != 0) return;
  TopkSmem sm(L.u);
  const uint64_t *staged = reinterpret_cast<const uint64_t *>(sm.lg);
  uint64_t k[1];
  k[0] = threadIdx.x < a.world * 64 ? staged[threadIdx.x] : 0ull;
  const uint64_t thr = block_kth_largest<1>(k, 64, sm.hist, sm.sh);
  collect_sorted64<1>(k, thr, sm.buf, sm.cnt, sm.sorted);
  topk_finish(a, sm.sorted);
}

// ---------------------------------------------------------------------------
// Before the grid barrier: everything the next phase can do without the previous
// phase's result -- its input's straddle list and the bulk copies of inputs that
// already exist -- then this thread-0 arrival on vbar (the first of two).
template <int R>
CH_DEV void pre_phase(const Phase &p, const MegaArgs &a, const StepParams &sp, const SmemLayout &L) {
  cp_async_wait_all();  // this phase's struct (copied two phases ago)
  fence_proxy_async();  // this thread's generic shared-memory writes before the bulk copies that reuse it
  __syncthreads();
  if (p.kind == PH_GEMV) {
    if ((p.pm == PM_NORM || p.pm == PM_ADD_NORM) && threadIdx.x == 0) {
      GemvStage S(L.u, p.K, p.pm);
      stage_copy(L, S.s1, p.x_in, p.K * 4);  // residual: written at least one barrier ago
      stage_copy(L, S.s3, p.norm_w, p.K * 4);
      if (p.post_w) stage_copy(L, S.s2, p.post_w, p.K * 4);
    }
  } else if (p.kind == PH_ATTN) {
    attn_pre<R>(p, a, sp, L);
  }
  __syncthreads();  // every expect_tx of this phase precedes the arrival
  if (threadIdx.x == 0) mbar_arrive(L.vbar);
}
// Right after the grid barrier (thread 0): bulk copies of the previous phase's
// output (and its straddle partials), then the second arrival on vbar.
template <int R>
CH_DEV void post_copies(const Phase &p, const MegaArgs &a, const StepParams &sp, const SmemLayout &L) {
  if (threadIdx.x != 0) return;
  if (p.kind == PH_GEMV && p.pm == PM_DIRECT && blockIdx.x == 0)  // the phase after ATTN: reset its counters
    for (uint32_t k = 0; k < a.nkv; k++) a.attn_counters[k] = 0u;
  fence_proxy_async_global();  // the other CTAs' generic writes, acquired by the barrier, before bulk reads
  if (p.kind == PH_GEMV) {
    GemvStage S(L.u, p.K, p.pm);
    if (p.pm == PM_DIRECT) stage_copy(L, S.s0, p.x_in, p.K * 4);
    if (p.pm == PM_ADD_NORM || p.pm == PM_GELU) {
      if (p.nsum <= 1) stage_copy(L, S.s0, p.r_in.direct, p.K * 4);  // act mode: K act values
      stage_copy(L, S.part, p.r_in.partial, gridDim.x * 32 * 4);
    }
  } else if (p.kind == PH_ATTN) {
    attn_post_copies<R>(p, a, sp, L);
  } else if (p.kind == PH_TOPK) {
    topk_post_copies(p, L);
  } else if (blockIdx.x == 0) {  // PH_MERGE: every rank's candidates, written by the peers before the barrier
    TopkSmem sm(L.u);
    stage_copy(L, sm.lg, a.xcand, a.world * 64 * 8);
  }
  mbar_arrive(L.vbar);
}

// R = q heads per kv head
template <int R>
__global__ void __launch_bounds__(MK_THREADS, 1) decode_step_kernel(const MegaArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  SmemLayout L;
  L.stages = smem;
  L.bars = reinterpret_cast<uint64_t *>(smem + MK_NW * MK_SPW * MK_STAGE);
  L.vbar = L.bars + MK_NW * MK_SPW;
  L.xzero = reinterpret_cast<uint4 *>(L.vbar + 2);
  L.wpart = reinterpret_cast<float *>(L.xzero + 1);
  L.sl = reinterpret_cast<uint32_t *>(L.wpart + MK_NW * 2 * 16);
  L.g4 = (gridDim.x + 3u) & ~3u;
  L.comb = reinterpret_cast<uint2 *>(L.sl + kKinds * 2 * L.g4);
  L.ncomb = reinterpret_cast<uint32_t *>(L.comb + kKinds * kMaxComb);
  L.wtab = reinterpret_cast<uint4 *>(L.ncomb + 8);
  L.wphys = reinterpret_cast<uint32_t *>(L.wtab + kKinds * MK_NW);
  L.u = reinterpret_cast<uint8_t *>(L.wphys + 2 * kWinSlots);
  __shared__ __align__(16) float red[32];
  __shared__ Phase ph_s[3];  // phases pi, pi+1 and pi+2 (copied ahead with cp.async)
  __shared__ StepParams sp_s;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t gw = blockIdx.x * MK_NW + warp;
  uint8_t *my_stages = L.stages + (size_t)warp * MK_SPW * MK_STAGE;
  uint64_t *my_bars = L.bars + warp * MK_SPW;
  const uint64_t pol = l2_evict_first_policy();
  Stream st;
  if (lane == 0) {
    for (int s = 0; s < MK_SPW; s++) mbar_init(&my_bars[s], 1);
    if (warp == 0) mbar_init(L.vbar, 2);
    fence_mbar_init();
    stream_init(a, gw, st);
    for (int s = 0; s < MK_SPW; s++)
      if (stream_next(a, gw, st)) stream_issue(st, my_stages + (size_t)s * MK_STAGE, &my_bars[s], pol);
  }
  if (threadIdx.x == 0) {
    *L.xzero = make_uint4(0u, 0u, 0u, 0u);
    sp_s = *a.sp;
    s_abort = (*(volatile uint32_t *)a.err & DEV_ERR_PEER_TIMEOUT) ? 1u : 0u;
    s_xep = a.base[2];
  }
  for (uint32_t i = 0; i < 2 && i < a.nphases; i++) copy_phase(a.phases + i, &ph_s[i]);
  cp_async_wait_all();
  __syncthreads();
  attn_lists_init(a, sp_s, L.wphys);
  launch_tables(a, L);
  pre_phase<R>(ph_s[0], a, sp_s, L);

  const unsigned long long base = a.base[0], gbase = a.base[1];  // arrivals before this launch
  TRACE_SMID();
  uint32_t cidx = 0, vpar = 0;
  bool ok = true;
  for (uint32_t pi = 0; pi < a.nphases; pi++) {
    const Phase &p = ph_s[pi % 3];
    PHASE_MARK(pi, 0);
    if (pi + 2 < a.nphases) copy_phase(a.phases + pi + 2, &ph_s[(pi + 2) % 3]);
    post_copies<R>(p, a, sp_s, L);
    if (!mbar_spin_bounded(L.vbar, vpar, a.err)) ok = false;
    vpar ^= 1u;
    PHASE_MARK(pi, 1);
    if (p.kind == PH_GEMV) {
      gemv_prologue(p, a, L, red, pi);
      __syncthreads();
      PHASE_MARK(pi, 2);
      const uint2 *xq = reinterpret_cast<const uint2 *>(L.u);
      const float *sxs = reinterpret_cast<const float *>(L.u) + p.K;
      if (p.pm == PM_DIRECT || p.pm == PM_GELU)  // Q4 o / down: f16 fragments
        gemv_tiles<FMT_Q4, false>(p, a, gw, L, xq, sxs, cidx, st, ok, pol, pi);
      else if (p.fmt == FMT_Q4)
        gemv_tiles<FMT_Q4, true>(p, a, gw, L, xq, sxs, cidx, st, ok, pol, pi);
      else
        gemv_tiles<FMT_Q8, true>(p, a, gw, L, xq, sxs, cidx, st, ok, pol, pi);
      __syncthreads();
      PHASE_MARK(pi, 3);
      cta_combine(p, a, L);
    } else if (p.kind == PH_ATTN) {
      attn_phase<R>(p, a, sp_s, L, pi);
    } else if (p.kind == PH_TOPK) {
      topk_phase(p, a, L);
    } else {
      merge_phase(a, L);
    }
#ifdef CH_PHASE_TRACE
    __syncthreads();
#endif
    PHASE_MARK(pi, 4);
    if (pi + 1 < a.nphases) {
      const bool cross = p.cross != 0;
      const unsigned long long ltarget = base + (unsigned long long)p.lidx * gridDim.x;
      if (p.nobar) {  // the consumers poll this phase's exchange words: no barrier
        __syncthreads();  // the CTA's stores are issued before its next phase reuses shared memory
        pre_phase<R>(ph_s[(pi + 1) % 3], a, sp_s, L);
        PHASE_MARK(pi, 5);
      } else {
        grid_arrive(a, cross, ltarget);
        pre_phase<R>(ph_s[(pi + 1) % 3], a, sp_s, L);
        PHASE_MARK(pi, 5);
        if (cross)
          grid_wait(a.garrive, true, gbase + (unsigned long long)p.gidx * a.world, a.err, &s_abort);
        else
          grid_wait(a.arrive, false, ltarget, a.err, &s_abort);
      }
      PHASE_MARK(pi, 6);
    }
  }
  if (!ok && lane == 0) {
    // a copy wait gave up: the last MK_SPW chunks' waits were skipped, so wait
    // (bounded) for those copies before the CTA exits
    for (uint32_t j = cidx >= MK_SPW ? cidx - MK_SPW : 0; j < cidx; j++)
      mbar_wait_bounded(&my_bars[j % MK_SPW], (j / MK_SPW) & 1, nullptr, 100000000ull);
  }
  // every CTA has passed the last barrier, so all have read `base`: advance it for the next launch
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    a.base[0] = base + (unsigned long long)a.nlocal * gridDim.x;
    a.base[1] = gbase + (unsigned long long)a.ncross * a.world;
    a.base[2] = s_xep + a.nx;
  }
}

size_t mk_smem_bytes(uint32_t max_k, uint32_t hidden, uint32_t ratio, uint32_t max_splits, uint32_t cache_slots,
                     uint32_t grid) {
  const size_t g4 = (grid + 3u) & ~3u;
  const size_t fixed = (size_t)MK_NW * MK_SPW * MK_STAGE + (MK_NW * MK_SPW + 2) * 8 + 16 + MK_NW * 2 * 16 * 4 +
                      kKinds * 2 * g4 * 4 + kKinds * kMaxComb * 8 + 8 * 4 + kKinds * MK_NW * 16 + 2 * kWinSlots * 4;
  const size_t part = (size_t)grid * 32 * 4;  // straddle partials of the previous GEMV
  // GEMV staging: 4 vectors of `hidden` for the norm prologues, one of max_k otherwise
  const size_t gemv = std::max((size_t)4 * hidden * 4, (size_t)max_k * 4) + part;
  const uint32_t chunk_cap = std::max(kMinChunk, (cache_slots + max_splits - 1) / max_splits);
  const size_t kv = (size_t)2 * kWinSlots * kHeadDim * 2, os = (size_t)MK_NW * ratio * kHeadDim * 4;
  const size_t attn = 4 * ((size_t)(ratio + 2) * kHeadDim + 2 * kHeadDim + kHeadDim) + std::max(kv, os) +
                      4 * ((size_t)ratio * chunk_cap + 2 * (size_t)ratio * max_splits + 2 * ratio) + 16 + part;
  const size_t topk = 256 * 4 + 32 + 128 * 8 + (4096 + 8) * 4 + part;
  return fixed + std::max({gemv, attn, topk});
}

template <int R>
static cudaError_t launch_decode_step_t(const MegaArgs &a, size_t smem, cudaStream_t s) {
  {
    const cudaError_t e = ensure_smem_attr((const void *)decode_step_kernel<R>, smem);
    if (e != cudaSuccess) return e;
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
  return cudaLaunchKernelEx(&cfg, decode_step_kernel<R>, a);
}

cudaError_t launch_decode_step(const MegaArgs &a, size_t smem, cudaStream_t s) {
  if (a.grid > kMaxGrid) return cudaErrorInvalidValue;
  switch (a.nq / a.nkv) {
    case 1: return launch_decode_step_t<1>(a, smem, s);
    case 2: return launch_decode_step_t<2>(a, smem, s);
    case 4: return launch_decode_step_t<4>(a, smem, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ch

#ifdef CH_PHASE_TRACE
// copies the timeline [cta][phase][mark] (u64 ns) of the last traced launch to host memory
extern "C" int ch_phase_trace_copy(unsigned long long *host, size_t count) {
  if (count > sizeof(ch::g_phase_trace) / 8) count = sizeof(ch::g_phase_trace) / 8;
  return cudaMemcpyFromSymbol(host, ch::g_phase_trace, count * 8) == cudaSuccess ? 0 : -3;
}
#endif
