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
