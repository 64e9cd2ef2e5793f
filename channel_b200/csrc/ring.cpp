// ring.cpp -- slot bookkeeping of the fixed 4,096-slot ring-buffer KV cache:
// DynamicRingBuffer (src/ring_buffer.zig:21-391), metadata only.  The K/V rows
// themselves live in each model's device cache ([4096][kv_dim] f16 per layer).
//
// Tiers (ring_buffer.zig:17-20): [0, anchors) immutable anchors, then a FIFO
// window up to recallStart = 4096 - 128, then 128 associative-recall slots.
// Slot lists come out in strict clock order (anchors, window, recall), which
// the attention kernels consume as gathered rows.
#include <algorithm>
#include <cstring>
#include <vector>

#include "../../include/channel_cuda.h"
#include "kernels.cuh"

namespace {
constexpr size_t kTotal = 4096, kRecall = 128, kMaxBoundaries = 1024;
}

struct ch_ring {
  size_t layers = 0, anchors = 0, ingested = 0;
  std::vector<size_t> clocks;
  std::vector<uint8_t> active;
  size_t boundary[kMaxBoundaries] = {};
  int btype[kMaxBoundaries] = {};
  float bsal[kMaxBoundaries] = {};
  size_t nb = 0;
};

static size_t recall_slots() { return kTotal < kRecall * 2 ? 0 : kRecall; }
static size_t recall_start() { return kTotal - recall_slots(); }

extern "C" ch_ring *ch_ring_create(uint32_t num_layers, uint32_t num_anchors) {
  ch_ring *r = new ch_ring();
  r->layers = num_layers;
  r->anchors = num_anchors;
  r->clocks.assign((size_t)num_layers * kTotal, 0);
  r->active.assign((size_t)num_layers * kTotal, 0);
  return r;
}
extern "C" void ch_ring_destroy(ch_ring *r) { delete r; }
extern "C" void ch_ring_reset(ch_ring *r) {
  std::fill(r->clocks.begin(), r->clocks.end(), 0);
  std::fill(r->active.begin(), r->active.end(), 0);
  r->ingested = 0;
  r->nb = 0;
}
extern "C" void ch_ring_set_num_anchors(ch_ring *r, size_t n) { r->anchors = std::min(n, kTotal - kRecall - 64); }
extern "C" size_t ch_ring_num_anchors(const ch_ring *r) { return r->anchors; }
extern "C" size_t ch_ring_total_ingested(const ch_ring *r) { return r->ingested; }
extern "C" size_t ch_ring_window_size(const ch_ring *r, size_t) {
  const size_t start = recall_start();
  return start > r->anchors ? start - r->anchors : 1;
}
extern "C" size_t ch_ring_get_slot_index(const ch_ring *r, size_t layer, size_t clock) {
  if (clock < r->anchors) return clock;
  return r->anchors + (clock - r->anchors) % ch_ring_window_size(r, layer);
}
extern "C" size_t ch_ring_activate_slot(ch_ring *r, size_t layer, size_t clock) {
  const size_t slot = ch_ring_get_slot_index(r, layer, clock), i = layer * kTotal + slot;
  r->clocks[i] = clock;
  r->active[i] = 1;
  if (layer == 0 && clock >= r->ingested) r->ingested = clock + 1;
  return slot;
}
extern "C" void ch_ring_activate_range(ch_ring *r, size_t clock0, size_t n, uint32_t *slots_out) {
  for (size_t c = clock0; c < clock0 + n; c++) {
    for (size_t l = 0; l < r->layers; l++) ch_ring_activate_slot(r, l, c);
    if (slots_out) slots_out[c - clock0] = (uint32_t)ch_ring_get_slot_index(r, 0, c);
  }
}
// One decode step's host work for n streams, each with its own ring: activate the clock's
// slot in layer 0, then the slot index and the full and sliding lists of layer 0 at that
// clock (forward.zig:42-45, per stream) straight into the step records and the caller's
// list storage (lists + b * 8192: active, then sliding).
extern "C" void ch_rings_fill_steps(ch_ring *const *rings, const uint32_t *streams, const uint32_t *tokens,
                                    const uint32_t *clocks, uint32_t n, size_t sliding_window, ch_stream_step *steps,
                                    uint32_t *lists) {
  for (uint32_t b = 0; b < n; b++) {
    ch_ring *r = rings[b];
    const size_t clock = clocks[b];
    ch_ring_activate_slot(r, 0, clock);
    uint32_t *act = lists + (size_t)b * 2 * kTotal, *sli = act + kTotal;
    ch_stream_step &st = steps[b];
    st.stream = streams[b];
    st.token = tokens[b];
    st.clock = (uint32_t)clock;
    st.slot = (uint32_t)ch_ring_get_slot_index(r, 0, clock);
    st.active = act;
    st.n_active = (uint32_t)ch_ring_active_slots(r, 0, clock, 0, sliding_window, act);
    st.sliding = sli;
    st.n_sliding = (uint32_t)ch_ring_active_slots(r, 0, clock, 1, sliding_window, sli);
  }
}
extern "C" void ch_ring_deactivate_slot(ch_ring *r, size_t layer, size_t clock) {
  const size_t i = layer * kTotal + ch_ring_get_slot_index(r, layer, clock);
  if (r->clocks[i] == clock) {
    r->active[i] = 0;
    r->clocks[i] = 0;
  }
}
extern "C" void ch_ring_rollback_clock(ch_ring *r, size_t target) {
  if (target >= r->ingested) return;
  for (size_t c = target; c < r->ingested; c++)
    for (size_t l = 0; l < r->layers; l++) ch_ring_deactivate_slot(r, l, c);
  r->ingested = target;
}
extern "C" void ch_ring_write_kv_meta(ch_ring *r, size_t layer, size_t clock) {
  const size_t i = layer * kTotal + ch_ring_get_slot_index(r, layer, clock);
  r->clocks[i] = clock;
  r->active[i] = 1;
  if (layer == 0 && clock >= r->ingested) r->ingested = clock + 1;
}
extern "C" void ch_ring_write_recall_meta(ch_ring *r, size_t layer, size_t rank, size_t clock) {
  const size_t slot = recall_start() + rank;
  if (slot >= kTotal) return;
  r->clocks[layer * kTotal + slot] = clock;
  r->active[layer * kTotal + slot] = 1;
}
extern "C" void ch_ring_clear_recall(ch_ring *r) {
  for (size_t l = 0; l < r->layers; l++)
    std::fill(r->active.begin() + l * kTotal + recall_start(), r->active.begin() + (l + 1) * kTotal, 0);
}
extern "C" void ch_ring_mark_boundary(ch_ring *r, size_t clock, int span_type, float salience) {
  if (r->nb > 0 && r->boundary[(r->nb - 1) % kMaxBoundaries] == clock) {
    r->btype[(r->nb - 1) % kMaxBoundaries] = span_type;
    r->bsal[(r->nb - 1) % kMaxBoundaries] = salience;
    return;
  }
  const size_t i = r->nb % kMaxBoundaries;
  r->boundary[i] = clock;
  r->btype[i] = span_type;
  r->bsal[i] = salience;
  r->nb++;
}
// first turn boundary at or after raw_min (ring_buffer.zig:92-100)
static size_t snap(const ch_ring *r, size_t raw_min) {
  if (raw_min <= r->anchors || r->nb == 0) return raw_min;
  for (size_t i = (r->nb > kMaxBoundaries ? r->nb - kMaxBoundaries : 0); i < r->nb; i++)
    if (r->boundary[i % kMaxBoundaries] >= raw_min) return r->boundary[i % kMaxBoundaries];
  return raw_min;
}
extern "C" int ch_ring_is_active(const ch_ring *r, size_t layer, size_t slot) { return r->active[layer * kTotal + slot]; }
extern "C" size_t ch_ring_slot_clock(const ch_ring *r, size_t layer, size_t slot) { return r->clocks[layer * kTotal + slot]; }

extern "C" size_t ch_ring_active_slots(const ch_ring *r, size_t layer, size_t clock, int is_sliding, size_t window,
                                       uint32_t *out) {
  const size_t base = layer * kTotal;
  const size_t eff = is_sliding ? window : ch_ring_window_size(r, layer);
  const size_t raw_min = clock >= eff ? clock - eff + 1 : 0;
  const size_t min_valid = is_sliding ? raw_min : snap(r, raw_min);
  size_t n = 0;
  for (size_t s = 0, lim = std::min(clock + 1, r->anchors); s < lim; s++)
    if (r->active[base + s] && (!is_sliding || s >= min_valid)) out[n++] = (uint32_t)s;
  for (size_t c = std::max(min_valid, r->anchors); c <= clock; c++) {
    const size_t slot = ch_ring_get_slot_index(r, layer, c);
    if (r->active[base + slot] && r->clocks[base + slot] == c) out[n++] = (uint32_t)slot;
  }
  if (!is_sliding)
    for (size_t s = recall_start(); s < kTotal; s++)
      if (r->active[base + s] && r->clocks[base + s] <= clock) out[n++] = (uint32_t)s;
  return n;
}

extern "C" size_t ch_ring_prefill_prev_slots(const ch_ring *r, size_t layer, size_t start_clock, size_t chunk_len,
                                             uint32_t *out) {
  if (start_clock == 0 || chunk_len == 0) return 0;
  const size_t base = layer * kTotal;
  const size_t end_clock = start_clock + chunk_len - 1, w = ch_ring_window_size(r, layer);
  const size_t min_valid = snap(r, end_clock >= w ? end_clock - w + 1 : 0);
  size_t n = 0;
  for (size_t s = 0, lim = std::min(start_clock, r->anchors); s < lim; s++)
    if (r->active[base + s]) out[n++] = (uint32_t)s;
  for (size_t c = std::max(min_valid, r->anchors); c < start_clock; c++) {
    const size_t slot = ch_ring_get_slot_index(r, layer, c);
    if (r->active[base + slot] && r->clocks[base + slot] == c) out[n++] = (uint32_t)slot;
  }
  for (size_t s = recall_start(); s < kTotal; s++)
    if (r->active[base + s] && r->clocks[base + s] < start_clock) out[n++] = (uint32_t)s;
  return n;
}

// Layer-0 metadata of a ring in the device layout (RingDevState) for the device-side
// list builder (ring_dev.cu); fails when a stored clock does not fit 32 bits.
namespace ch {
bool ring_export_layer0(const ch_ring *r, RingDevState *out) {
  out->anchors = (uint32_t)r->anchors;
  out->window = (uint32_t)ch_ring_window_size(r, 0);
  if (r->nb > 0xFFFFFFFFull || r->ingested > 0xFFFFFFFFull) return false;
  out->nb = (uint32_t)r->nb;
  out->ingested = (uint32_t)r->ingested;
  out->next_clock = 0;
  out->step = 0;
  out->pad0 = out->pad1 = 0;
  for (size_t s = 0; s < kTotal; s++) {
    if (r->clocks[s] > 0xFFFFFFFFull) return false;
    out->clocks[s] = (uint32_t)r->clocks[s];
    out->active[s] = r->active[s];
  }
  for (size_t i = 0; i < kMaxBoundaries; i++) {
    if (r->boundary[i] > 0xFFFFFFFFull) return false;
    out->boundary[i] = (uint32_t)r->boundary[i];
  }
  return true;
}
}  // namespace ch
