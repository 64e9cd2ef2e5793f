"""Ragged multi-stream greedy decode over one model.

Each stream has its own ring (host bookkeeping, ``DynamicRingBuffer``) and its own
4,096-slot KV cache per layer on the device.  Prompts of any length are prefilled
stream by stream (batched tcgen05 GEMMs + causal attention into that stream's
cache); then every step packs one token from each unfinished stream -- up to
``max_batch`` per launch -- into ``ch_streams_decode``: the weights are read once
per step for the whole batch, and each token attends to its own stream's cache at
its own position.  The per-stream host work per step is the same as the
single-stream engine's (``src/model/forward.zig:42-45``: activate the clock's slot,
read the active and sliding lists); the reference itself serves one stream
(``src/server_queue.zig:9-145``), so the packing is new.
"""
from __future__ import annotations

import ctypes as C
from typing import List, Sequence

import numpy as np

from . import _lib as L
from .engine import DynamicRingBuffer

_u32p = C.POINTER(C.c_uint32)


class MultiStreamDecoder:
    def __init__(self, gm, config, n_streams: int, max_batch: int):
        self.gm, self.cfg = gm, config
        self.n, self.max_batch = n_streams, max_batch
        gm.streams_init(n_streams, max_batch)
        self.rings = [DynamicRingBuffer(config.num_hidden_layers, 0) for _ in range(n_streams)]
        self.clock = [0] * n_streams
        self.next_token = [0] * n_streams
        self.tokens: List[List[int]] = [[] for _ in range(n_streams)]
        self.steps = 0  # batched decode launches so far
        # step records and list storage reused by every step (ch_rings_fill_steps)
        self._step_recs = (L.ChStreamStep * max_batch)()
        self._lists = np.empty(max_batch * 2 * 4096, np.uint32)

    def prefill(self, stream: int, prompt: Sequence[int]) -> int:
        """Prefill the stream's prompt from clock 0, in chunks of at most the model's
        max_prefill_tokens (each chunk attends to the earlier ones through the ring's
        previous slots); returns (and records) its first greedy token."""
        ring, n = self.rings[stream], len(prompt)
        cap = self.cfg.max_prefill_tokens
        prompt = np.asarray(prompt, np.uint32)
        tok = 0
        for c0 in range(0, n, cap):
            m = min(cap, n - c0)
            prev = ring.getPrefillPrevSlots(0, c0, m)
            slots = np.concatenate([prev, ring.activateRange(c0, m)]).astype(np.uint32)
            tok = self.gm.stream_prefill(stream, prompt[c0:c0 + m], slots, c0, len(prev))
        self.clock[stream], self.next_token[stream], self.tokens[stream] = n, tok, [tok]
        return tok

    def _step_lists(self, stream: int):
        ring, clock, w = self.rings[stream], self.clock[stream], self.cfg.sliding_window
        ring.activateSlot(0, clock)
        return (ring.getSlotIndex(clock), ring.getActiveSlotsLayer(0, clock, False, w),
                ring.getActiveSlotsLayer(0, clock, True, w))

    def step(self, streams: Sequence[int]) -> np.ndarray:
        """One batched greedy step over distinct streams (<= max_batch); returns their next
        tokens.  The per-stream ring work of _step_lists runs in one C call for the batch."""
        n = len(streams)
        if n > self.max_batch:
            raise ValueError("more streams than max_batch in one step")
        ids = np.asarray(streams, np.uint32)
        tokens = np.array([self.next_token[s] for s in streams], np.uint32)
        clocks = np.array([self.clock[s] for s in streams], np.uint32)
        rings = (C.c_void_p * n)(*[self.rings[s].h for s in streams])
        L.load().ch_rings_fill_steps(rings, ids.ctypes.data_as(_u32p), tokens.ctypes.data_as(_u32p),
                                     clocks.ctypes.data_as(_u32p), n, self.cfg.sliding_window, self._step_recs,
                                     self._lists.ctypes.data_as(_u32p))
        out = self.gm.streams_decode_steps(self._step_recs, n)
        for s, t in zip(streams, out):
            self.next_token[s] = int(t)
            self.tokens[s].append(int(t))
            self.clock[s] += 1
        self.steps += 1
        return out

    def run(self, prompts: Sequence[Sequence[int]], n_tokens: int) -> List[List[int]]:
        """Prefill every stream, then decode until each has n_tokens greedy tokens
        (the prefill's token counts as the first).  Streams are packed up to
        max_batch per step, in stream order."""
        for s, p in enumerate(prompts):
            self.prefill(s, p)
        while True:
            live = [s for s in range(len(prompts)) if len(self.tokens[s]) < n_tokens]
            if not live:
                break
            for i in range(0, len(live), self.max_batch):
                self.step(live[i:i + self.max_batch])
        return [t[:n_tokens] for t in self.tokens[:len(prompts)]]
