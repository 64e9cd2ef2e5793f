"""Ring lists built on the device (ch_ring_dev_*) against the host ring
(DynamicRingBuffer restatement, src/ring_buffer.zig:287-380), bit for bit and in
order: the reference's own ring known-answer scenarios, random histories (anchors,
wrap-around, turn boundaries, recall slots, rollbacks), the activation the decode
loop does on the device, prefill-previous lists -- and the device-ring decode loop
(ch_decode_run_ring) against the planned loop and the oracle's greedy stream."""
import ctypes as C
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from channel_b200 import _lib as L
from channel_b200.engine import DynamicRingBuffer
from tests.gpu_util import call

pytestmark = pytest.mark.gpu
KATS = json.loads((Path(__file__).parent / "golden" / "reference_kats.json").read_text())


class DevRing:
    def __init__(self, ctx):
        self.lib = L.load()
        h = C.c_void_p()
        L.check(self.lib.ch_ring_dev_create(ctx.handle, C.byref(h)))
        self.h = h.value
        self.ctx = ctx
        self.buf = torch.zeros(2 * 4096 + 4, dtype=torch.int32, device="cuda")

    def upload(self, ring):
        L.check(self.lib.ch_ring_dev_upload(self.h, ring.h))

    def lists(self, clock, window, activate=False):
        b = self.buf
        p = b.data_ptr()
        call(self.lib.ch_ring_dev_lists, self.h, clock, int(activate), window, p + 4 * 8192, p, p + 4 * 8193,
             p + 4 * 4096, p + 4 * 8194)
        self.ctx.synchronize()
        a = b.cpu().numpy().view(np.uint32)
        return int(a[8192]), a[:a[8193]].copy(), a[4096:4096 + a[8194]].copy()

    def prev(self, start, n):
        p = self.buf.data_ptr()
        call(self.lib.ch_ring_dev_prefill_prev, self.h, start, n, p, p + 4 * 8193)
        self.ctx.synchronize()
        a = self.buf.cpu().numpy().view(np.uint32)
        return a[:a[8193]].copy()

    def close(self):
        self.lib.ch_ring_dev_destroy(self.h)


def _check_clock(dr, ring, clock, window):
    _, act, sli = dr.lists(clock, window)
    np.testing.assert_array_equal(act, ring.getActiveSlotsLayer(0, clock, False, window), err_msg=f"full @ {clock}")
    np.testing.assert_array_equal(sli, ring.getActiveSlotsLayer(0, clock, True, window), err_msg=f"sliding @ {clock}")


def test_reference_ring_kats_on_device(ctx):
    from tests.test_reference_kats import ProductRingAdapter, run_ops
    dr = DevRing(ctx)
    try:
        n_checked = 0
        for kat in KATS["ring"]:
            r = ProductRingAdapter(*kat["init"])
            stage = kat
            while stage:  # a case and its follow-up stages ("then")
                run_ops(r, stage["ops"])
                dr.upload(r.r)
                for chk in stage["checks"]:
                    name, *a = chk
                    if name in ("active_count", "active_at") and a[0] == 0:
                        layer, clock, sl, w = a[:4]
                        _, act, sli = dr.lists(clock, w)
                        got = sli if sl else act
                        np.testing.assert_array_equal(got, r.lst(0, clock, sl, w), err_msg=kat["name"])
                        if name == "active_count":
                            assert len(got) == a[4], (kat["name"], chk)
                        else:
                            assert int(got[a[4]]) == a[5], (kat["name"], chk)
                        n_checked += 1
                    elif name == "prefill_prev_bounds" and a[0] == 0:
                        _, start, chunk, _ = a
                        np.testing.assert_array_equal(dr.prev(start, chunk), r.prev(0, start, chunk),
                                                      err_msg=kat["name"])
                        n_checked += 1
                stage = stage.get("then")
        assert n_checked >= 3
    finally:
        dr.close()


@pytest.mark.parametrize("seed", [0, 1, 2, 3])
def test_random_histories_match_host_ring(ctx, seed):
    rng = np.random.default_rng(seed)
    anchors = [0, 4, 512, 3900][seed]
    ring = DynamicRingBuffer(2, anchors)
    dr = DevRing(ctx)
    try:
        clock = 0
        for phase in range(5):
            n = int(rng.integers(50, 3000))
            for c in range(clock, clock + n):
                ring.activateSlot(0, c)
                if rng.random() < 0.02:
                    ring.markBoundary(c, 6, 1.0)
            clock += n
            if rng.random() < 0.5:  # associative recall slots
                for rank in range(int(rng.integers(1, 128))):
                    ring.writeRecallKV(0, rank, int(rng.integers(0, clock + 10)))
            if phase == 2 and rng.random() < 0.7:  # roll back part of the history
                clock -= int(rng.integers(1, min(clock, 700)))
                ring.rollbackClock(clock)
            dr.upload(ring)
            for w in (1, 8, 1024, 5000):
                _check_clock(dr, ring, max(clock - 1, 0), w)
            for c in rng.integers(0, clock + 50, 4):
                _check_clock(dr, ring, int(c), 1024)
            for start, m in [(clock, 17), (max(clock - 300, 0), 300), (int(rng.integers(1, clock + 1)), 1024)]:
                np.testing.assert_array_equal(dr.prev(start, m), ring.getPrefillPrevSlots(0, start, m),
                                              err_msg=f"prefill prev {start}+{m}")
            # the device loop's own step: activate the next clock, then both lists
            slot, act, sli = dr.lists(clock, 1024, activate=True)
            ring.activateSlot(0, clock)
            assert slot == ring.getSlotIndex(clock)
            np.testing.assert_array_equal(act, ring.getActiveSlotsLayer(0, clock, False, 1024))
            np.testing.assert_array_equal(sli, ring.getActiveSlotsLayer(0, clock, True, 1024))
            clock += 1
    finally:
        dr.close()
        ring.deinit()


def test_decode_run_ring_matches_planned_loop_and_oracle(ctx, oracle):
    from channel_b200 import GpuModelContext
    from tests.model_util import ring_step_lists, small_config
    cfg = small_config()
    gm = GpuModelContext.synthetic(ctx, cfg, 5)
    w = oracle.SyntheticWeights(cfg, 5)
    om = oracle.Model(cfg, w)
    lib = L.load()
    dr = DevRing(ctx)
    n = 24
    try:
        # oracle greedy stream from clock 0
        ring_o = DynamicRingBuffer(cfg.num_hidden_layers, 0)
        tok, ref = 9, []
        for clock in range(n):
            slot, act, sli = ring_step_lists(ring_o, cfg, clock)
            tok, _, _ = om.forward_token(oracle.embed(w.embed, [int(tok)], cfg.hidden_size)[0], clock, slot, act, sli)
            ref.append(int(tok))
        # device ring loop
        gm.zero_state()
        ring = DynamicRingBuffer(cfg.num_hidden_layers, 0)
        dr.upload(ring)
        L.check(lib.ch_decode_run_ring(gm.handle, dr.h, ring.h, 9, 0, n))
        got = [int(t) for t in gm.decode_tokens(n)]
        assert got == ref, (got, ref)
        # the host ring took the same activations
        for clock in range(n):
            assert ring.is_active(0, ring.getSlotIndex(clock)) and ring.slot_clock(0, ring.getSlotIndex(clock)) == clock
        # planned loop on the same model and clocks agrees
        gm.zero_state()
        ring2 = DynamicRingBuffer(cfg.num_hidden_layers, 0)
        gm.decode_plan([(c, *ring_step_lists(ring2, cfg, c)) for c in range(n)])
        gm.decode_run(9, n)
        assert [int(t) for t in gm.decode_tokens(n)] == ref
        assert ctx.device_status() == 0
    finally:
        dr.close()
        gm.deinit()
