"""ch_ring_activate_range (one call for a prompt chunk's ring bookkeeping) leaves the
ring exactly as per-slot activateSlot calls in every layer do, and returns the
layer-0 slots (host only)."""
import numpy as np

from channel_b200 import DynamicRingBuffer


def test_activate_range_matches_per_slot():
    layers, window = 3, 16
    a, b = DynamicRingBuffer(layers, 2), DynamicRingBuffer(layers, 2)
    for c0, n in [(0, 7), (7, 4200), (4207, 5)]:  # wraps the 4,096-slot window
        got = a.activateRange(c0, n)
        want = []
        for c in range(c0, c0 + n):
            for layer in range(layers):
                b.activateSlot(layer, c)
            want.append(b.getSlotIndex(c))
        assert np.array_equal(got, np.asarray(want, np.uint32))
        clock = c0 + n - 1
        for layer in range(layers):
            for sliding in (False, True):
                assert np.array_equal(a.getActiveSlotsLayer(layer, clock, sliding, window),
                                      b.getActiveSlotsLayer(layer, clock, sliding, window))


def test_rings_fill_steps_matches_per_call():
    """ch_rings_fill_steps (one decode step's ring work for many streams) writes the
    records the per-call path builds: slot, full and sliding lists of layer 0 after
    activating the clock's slot, for rings at different clocks (past the 4,096-slot wrap
    and the sliding window)."""
    import ctypes as C
    from channel_b200 import _lib as L
    lib = L.load()
    u32p = C.POINTER(C.c_uint32)
    layers, window = 3, 64
    starts = [5, 700, 4090, 5000, 12]
    a = [DynamicRingBuffer(layers, 1) for _ in starts]
    b = [DynamicRingBuffer(layers, 1) for _ in starts]
    for ra, rb, c in zip(a, b, starts):
        ra.activateRange(0, c)
        rb.activateRange(0, c)
    streams = np.array([3, 0, 4, 1, 2], np.uint32)  # any stream ids, step order kept
    tokens = np.array([11, 22, 33, 44, 55], np.uint32)
    for step in range(3):
        clocks = np.array([c + step for c in starts], np.uint32)
        n = len(a)
        recs = (L.ChStreamStep * n)()
        lists = np.empty(n * 2 * 4096, np.uint32)
        rings = (C.c_void_p * n)(*[r.h for r in a])
        lib.ch_rings_fill_steps(rings, streams.ctypes.data_as(u32p), tokens.ctypes.data_as(u32p),
                                clocks.ctypes.data_as(u32p), n, window, recs, lists.ctypes.data_as(u32p))
        for i, (rb, clock) in enumerate(zip(b, clocks)):
            clock = int(clock)
            rb.activateSlot(0, clock)
            r = recs[i]
            assert (r.stream, r.token, r.clock) == (int(streams[i]), int(tokens[i]), clock)
            assert r.slot == rb.getSlotIndex(clock)
            act = np.ctypeslib.as_array(r.active, shape=(r.n_active,))
            sli = np.ctypeslib.as_array(r.sliding, shape=(r.n_sliding,))
            assert np.array_equal(act, rb.getActiveSlotsLayer(0, clock, False, window))
            assert np.array_equal(sli, rb.getActiveSlotsLayer(0, clock, True, window))
            assert r.n_sliding <= window + 1  # the window really trims
