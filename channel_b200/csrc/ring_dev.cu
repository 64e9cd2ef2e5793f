// ring_dev.cu -- the ring buffer's slot lists generated on the device.
//
// The reference builds the decode step's slot lists on the host every token
// (DynamicRingBuffer.getActiveSlotsLayer, src/ring_buffer.zig:287-339, called
// from forward.zig:44-45) and uploads them (model_dispatch.zig:133-135).  Here a
// device copy of the ring's layer-0 metadata -- active flags, the clock each slot
// holds, the anchor count and the turn boundaries -- lets one CTA activate the
// step's slot and build both lists (full window with boundary snapping and
// recall slots; sliding window) in the reference's order, so a device-resident
// decode loop needs no host work and no upload per token.
//
// List construction is a stream compaction over the candidates in the order the
// reference visits them (anchors, then the window clocks oldest first, then the
// recall slots): each thread tests 4 consecutive candidates, a block-wide
// exclusive scan of the keep counts gives every kept slot its output position.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.cuh"

namespace ch {

namespace {
constexpr int kRdThreads = 1024;
constexpr uint32_t kCandPerThread = 4;
constexpr uint32_t kCandPerRound = kRdThreads * kCandPerThread;

CH_DEV uint32_t rd_slot(const RingDevState &r, uint32_t clock) {
  if (clock < r.anchors) return clock;
  return r.anchors + (clock - r.anchors) % r.window;  // window = windowSize(0) (ring_buffer.zig:110-113)
}

// first turn boundary (insertion order) at or after raw_min, else raw_min (snapToBoundary,
// ring_buffer.zig:86-99).  Whole block; `s_min` is shared scratch.
CH_DEV uint32_t rd_snap(const RingDevState &r, uint32_t raw_min, uint32_t *s_min) {
  if (raw_min <= r.anchors || r.nb == 0) return raw_min;
  const uint32_t start = r.nb > kRingMaxBoundaries ? r.nb - kRingMaxBoundaries : 0;
  if (threadIdx.x == 0) *s_min = 0xFFFFFFFFu;
  __syncthreads();
  for (uint32_t i = start + threadIdx.x; i < r.nb; i += blockDim.x)
    if (r.boundary[i % kRingMaxBoundaries] >= raw_min) atomicMin(s_min, i);
  __syncthreads();
  const uint32_t first = *s_min;
  __syncthreads();
  return first == 0xFFFFFFFFu ? raw_min : r.boundary[first % kRingMaxBoundaries];
}

// exclusive block scan of v (kRdThreads threads); total in *s_total
CH_DEV uint32_t block_excl_scan(uint32_t v, uint32_t *s_warp, uint32_t *s_total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < kRdThreads / 32 ? s_warp[lane] : 0u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    s_warp[lane] = w;  // inclusive prefix over warps
    if (lane == 31) *s_total = w;
  }
  __syncthreads();
  const uint32_t before = warp ? s_warp[warp - 1] : 0u;
  const uint32_t r = before + x - v;
  __syncthreads();
  return r;
}

// One list (getActiveSlotsLayer(0, clock, is_sliding, window) or, prev = true,
// getPrefillPrevSlots(0, clock = start_clock, chunk_len)) into out; returns its length.
CH_DEV uint32_t rd_list(const RingDevState &r, uint32_t clock, bool is_sliding, uint32_t sliding_window, bool prev,
                        uint32_t chunk_len, uint32_t *out, uint32_t *sh) {
  uint32_t *s_min = sh, *s_total = sh + 1, *s_warp = sh + 2;
  uint32_t min_valid, lim_a, ds, n_b, c_b0, recall_bound;
  if (prev) {  // ring_buffer.zig:341-380: clocks before start_clock of a chunk ending at clock + chunk_len - 1
    const uint32_t end_clock = clock + chunk_len - 1;
    const uint32_t raw_min = end_clock >= r.window ? end_clock - r.window + 1 : 0;
    min_valid = rd_snap(r, raw_min, s_min);
    lim_a = min(clock, r.anchors);
    ds = max(min_valid, r.anchors);
    n_b = clock > ds ? clock - ds : 0;
    recall_bound = clock;  // recall slots with clock < start_clock
  } else {
    const uint32_t eff = is_sliding ? sliding_window : r.window;
    const uint32_t raw_min = clock >= eff ? clock - eff + 1 : 0;
    min_valid = is_sliding ? raw_min : rd_snap(r, raw_min, s_min);
    lim_a = min(clock + 1, r.anchors);
    ds = max(min_valid, r.anchors);
    n_b = clock >= ds ? clock - ds + 1 : 0;
    recall_bound = clock + 1;  // recall slots with clock <= curr_clock
  }
  c_b0 = ds;
  const uint32_t n_c = (is_sliding && !prev) ? 0u : kRingSlots - kRingRecallStart;
  const uint32_t total = lim_a + n_b + n_c;
  uint32_t base = 0;
  for (uint32_t r0 = 0; r0 < total; r0 += kCandPerRound) {
    uint32_t slot[kCandPerThread], keep = 0;
#pragma unroll
    for (uint32_t j = 0; j < kCandPerThread; j++) {
      const uint32_t i = r0 + threadIdx.x * kCandPerThread + j;
      bool k = false;
      uint32_t s = 0;
      if (i < lim_a) {  // 1. anchors: clock = slot
        s = i;
        k = r.active[s] && (!is_sliding || prev || s >= min_valid);
      } else if (i < lim_a + n_b) {  // 2. the window, oldest clock first
        const uint32_t c = c_b0 + (i - lim_a);
        s = rd_slot(r, c);
        k = r.active[s] && r.clocks[s] == c;
      } else if (i < total) {  // 3. recall slots
        s = kRingRecallStart + (i - lim_a - n_b);
        k = r.active[s] && r.clocks[s] < recall_bound;
      }
      slot[j] = s;
      keep |= (k ? 1u : 0u) << j;
    }
    const uint32_t pos = base + block_excl_scan(__popc(keep), s_warp, s_total);
    uint32_t p = pos;
#pragma unroll
    for (uint32_t j = 0; j < kCandPerThread; j++)
      if (keep >> j & 1u) out[p++] = slot[j];
    base += *s_total;
    __syncthreads();
  }
  return base;
}

__global__ void __launch_bounds__(kRdThreads, 1) ring_step_kernel(const RingStepArgs a) {
  __shared__ uint32_t sh[2 + kRdThreads / 32];
  RingDevState &r = *a.ring;
  uint32_t clock = a.clock;
  if (a.loop) clock = r.next_clock;  // device loop: the ring's own clock
  if (a.activate && threadIdx.x == 0) {  // activateSlot(0, clock) (ring_buffer.zig:121-129)
    const uint32_t s = rd_slot(r, clock);
    r.clocks[s] = clock;
    r.active[s] = 1;
    if (clock >= r.ingested) r.ingested = clock + 1;
  }
  __syncthreads();
  if (a.prev) {
    const uint32_t n = rd_list(r, clock, false, 0, true, a.chunk_len, a.active_out, sh);
    if (threadIdx.x == 0) *a.n_active_out = n;
    return;
  }
  const uint32_t na = rd_list(r, clock, false, a.sliding_window, false, 0, a.active_out, sh);
  const uint32_t ns = rd_list(r, clock, true, a.sliding_window, false, 0, a.sliding_out, sh);
  if (threadIdx.x == 0) {
    const uint32_t slot = rd_slot(r, clock);
    if (a.slot_out) *a.slot_out = slot;
    if (a.n_active_out) *a.n_active_out = na;
    if (a.n_sliding_out) *a.n_sliding_out = ns;
    if (a.sp) {  // the decode step's parameters, like step_begin's plan entry
      StepParams p{};
      p.clock = clock;
      p.slot = slot;
      p.n_active = na;
      p.n_sliding = ns;
      p.active = a.active_out;
      p.sliding = a.sliding_out;
      p.step = r.step;
      p.next = 0;
      p.force = 0;
      *a.sp = p;
    }
    if (a.loop) {
      r.next_clock = clock + 1;
      r.step++;
    }
  }
}
}  // namespace

cudaError_t launch_ring_step(const RingStepArgs &a, cudaStream_t s) {
  ring_step_kernel<<<1, kRdThreads, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace ch
