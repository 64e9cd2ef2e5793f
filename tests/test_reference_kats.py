"""The reference's own known-answer tests (tests/golden/reference_kats.json,
transcribed from src/ring_buffer.zig, src/sampler.zig and src/tensor.zig test
blocks) run against the oracle AND against the product's C++ ring."""
import json
from pathlib import Path

import numpy as np
import pytest

KATS = json.loads((Path(__file__).parent / "golden" / "reference_kats.json").read_text())


class OracleRingAdapter:
    def __init__(self, o, layers, anchors):
        self.r = o.Ring(layers, anchors)
        self.o = o

    def writeKV(self, l, c): self.r.write_kv_meta(l, c)
    def writeRecallKV(self, l, rank, c): self.r.write_recall_meta(l, rank, c)
    def clearRecall(self): self.r.clear_recall()
    def activate(self, l, c): self.r.activate_slot(l, c)
    def rollbackClock(self, t): self.r.rollback_clock(t)
    def slot(self, l, c): return self.r.get_slot_index(l, c)
    def active(self, l, s): return bool(self.r.is_active(l, s))
    def clock_of(self, l, s): return self.r.slot_clock(l, s)
    def total(self): return self.r.total_ingested()
    def lst(self, l, c, sl, w): return self.r.active_list(l, c, sl, w)
    def prev(self, l, s, n): return self.r.prefill_prev(l, s, n)


class ProductRingAdapter:
    def __init__(self, layers, anchors):
        from channel_b200.engine import DynamicRingBuffer
        self.r = DynamicRingBuffer(layers, anchors)

    def writeKV(self, l, c): self.r.writeKV(l, c)
    def writeRecallKV(self, l, rank, c): self.r.writeRecallKV(l, rank, c)
    def clearRecall(self): self.r.clearRecall()
    def activate(self, l, c): self.r.activateSlot(l, c)
    def rollbackClock(self, t): self.r.rollbackClock(t)
    def slot(self, l, c): return self.r.getSlotIndexLayer(l, c)
    def active(self, l, s): return self.r.is_active(l, s)
    def clock_of(self, l, s): return self.r.slot_clock(l, s)
    def total(self): return self.r.total_ingested
    def lst(self, l, c, sl, w): return self.r.getActiveSlotsLayer(l, c, sl, w)
    def prev(self, l, s, n): return self.r.getPrefillPrevSlots(l, s, n)


def run_ops(r, ops):
    for op in ops:
        name, *a = op
        if name == "activate_write":
            layer, n = a
            for c in range(n):
                r.activate(layer, c)
                r.writeKV(layer, c)
        elif name == "activate_range":
            c0, c1, nl = a
            for c in range(c0, c1):
                for l in range(nl):
                    r.activate(l, c)
        elif name == "recordAttention":
            r.r.record_attention(*a)
        elif name == "recordAttentionClock":
            l, c, m = a
            r.r.record_attention(l, r.slot(0, c), m)
        else:
            getattr(r, name)(*a)


def run_checks(r, checks):
    for chk in checks:
        name, *a = chk
        if name == "active_count":
            l, c, sl, w, n = a
            assert len(r.lst(l, c, sl, w)) == n, chk
        elif name == "active_at":
            l, c, sl, w, i, v = a
            assert int(r.lst(l, c, sl, w)[i]) == v, chk
        elif name == "prefill_prev_bounds":
            l, start, chunk, min_anchors = a
            prev = r.prev(l, start, chunk)
            assert len(prev) + chunk <= 4096
            assert len(prev) >= min_anchors
            clocks = [r.clock_of(l, int(s)) for s in prev]
            assert all(b > a_ for a_, b in zip(clocks, clocks[1:])), "prev slots must be in strictly increasing clock order"
        elif name == "total_ingested":
            assert r.total() == a[0], chk
        elif name == "slot_active_of_clock":
            l, c, want = a
            assert r.active(l, r.slot(l, c)) == want, chk
        elif name == "mass_eq":
            l, s, v = a
            assert r.r.attention_mass(l, s) == np.float32(v)
        elif name == "salience_eq":
            s, v = a
            assert r.r.slot_salience(s) == np.float32(v)
        elif name == "evict":
            lo, hi, n, want = a
            assert r.r.evict_low_salience(lo, hi, n) == want
        elif name == "gini_lt":
            assert r.r.working_set_gini() < a[0]
        elif name == "gini_gt":
            assert r.r.working_set_gini() > a[0]
        elif name == "saturated":
            cap, g, want = a
            assert bool(r.r.is_saturated(cap, g)) == want
        else:
            raise AssertionError(f"unknown check {name}")


def run_case(r, case):
    run_ops(r, case["ops"])
    run_checks(r, case["checks"])
    nxt = case.get("then")
    while nxt:
        run_ops(r, nxt["ops"])
        run_checks(r, nxt["checks"])
        nxt = nxt.get("then")


@pytest.mark.parametrize("case", KATS["ring"] + KATS["ring_oracle_only"], ids=lambda c: c["name"][:48])
def test_ring_kat_oracle(oracle, case):
    run_case(OracleRingAdapter(oracle, *case["init"]), case)


@pytest.mark.parametrize("case", KATS["ring"], ids=lambda c: c["name"][:48])
def test_ring_kat_product(case):
    run_case(ProductRingAdapter(*case["init"]), case)


@pytest.mark.parametrize("case", KATS["sampler"], ids=lambda c: c["name"][:48])
def test_sampler_kat_oracle(oracle, case):
    ids = np.array([c[0] for c in case["cands"]], np.uint32)
    vals = np.array([c[1] for c in case["cands"]], np.float32)
    rec = None if case["recent"] is None else np.array(case["recent"], np.uint32)
    got = oracle.lib().or_sample_topk_greedy(
        oracle.p(ids, oracle.u32), oracle.p(vals, oracle.f32), len(ids),
        None if rec is None else oracle.p(rec, oracle.u32), 0 if rec is None else len(rec),
        case["repeat"], case["freq"], case["pres"], case["think"], case["close"], case["crit"])
    assert got == case["expect"]


def test_bf16_roundtrip_kat(oracle):
    l = oracle.lib()
    for v, tol in KATS["bf16"]["cases"]:
        back = l.or_bf16_to_f32(l.or_bf16_from_f32(v))
        assert abs(back - v) <= tol
    assert l.or_bf16_to_f32(l.or_bf16_from_f32(0.0)) == 0.0


@pytest.mark.parametrize("case", KATS["sampler"], ids=lambda c: c["name"][:48])
def test_sampler_kat_full_sampler_at_temp_zero(oracle, case):
    """the same known answers through the full sampleTopK restatement (temp 0)"""
    s = oracle.Sampler(42, 0.0, 0.95, repeat_penalty=case["repeat"], frequency_penalty=case["freq"],
                       presence_penalty=case["pres"], suppress_thinking=bool(case["think"]),
                       suppress_critique=bool(case["crit"]), suppress_channel_close=bool(case["close"]))
    ids = [c[0] for c in case["cands"]]
    vals = [c[1] for c in case["cands"]]
    assert s.sample_topk(ids, vals, case["recent"]) == case["expect"]


def test_sampler_kat_low_temperature(oracle):
    """src/sampler.zig:448-452: Sampler.init(42, 0.01, 0.95), repeat_penalty 1.2, recent
    [4373, 4373] over the three candidates of :437-441 -> 705"""
    s = oracle.Sampler(42, 0.01, 0.95, repeat_penalty=1.2)
    assert s.sample_topk([4373, 705, 1980], [18.0, 17.5, 16.0], [4373, 4373]) == 705
