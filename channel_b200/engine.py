"""Host-side mirror of the reference's GPU dispatch interface over the C-ABI.

Names and argument meaning follow Sullux/channel's Zig modules so callers and
tests read like the reference:

    GpuContext.init / deinit                 src/gpu/context.zig:17,109
    GpuModelContext.init / deinit            src/gpu/model_gpu.zig:68,203
    gpu_dispatch_forward_token               src/gpu/model_dispatch.zig:128
    gpu_dispatch_prefill_batch               src/gpu/batch_dispatch.zig:27
    DynamicRingBuffer                        src/ring_buffer.zig:21
    ModelConfig / TopKCandidate              src/model/types.zig:43,115

Errors: every failing call raises ChannelError carrying the C status
(the reference returns token 0 from a failed decode submit,
model_dispatch.zig:144, and raises BatchTooLarge / GpuError from prefill).
"""
from __future__ import annotations

import ctypes as C
from collections import abc as _abc
from dataclasses import dataclass, field
from typing import Callable, Optional, Sequence

import numpy as np

from . import _lib as L

TOTAL_SLOTS = 4096
UPPER_RECALL_SLOTS = 128


_PTR_TYPES: dict = {}


def _ptr(a: Optional[np.ndarray], ct):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    pt = _PTR_TYPES.get(ct)
    if pt is None:
        pt = _PTR_TYPES[ct] = C.POINTER(ct)
    return C.cast(a.ctypes.data, pt)  # cheaper than ndarray.ctypes.data_as per call


@dataclass
class TopKCandidate:
    id: int = 0
    val: float = 0.0


class TopKList(_abc.Sequence):
    """The 64 TopKCandidate of a step, read from the C-ABI result array on access (a
    decode loop that only wants the token does not pay for 64 Python objects)."""

    __slots__ = ("_tk",)

    def __init__(self, tk):
        self._tk = tk

    def __len__(self) -> int:
        return len(self._tk)

    def __getitem__(self, i):
        if isinstance(i, slice):
            return [TopKCandidate(t.id, t.val) for t in self._tk[i]]
        t = self._tk[i]
        return TopKCandidate(t.id, t.val)

    def __eq__(self, other) -> bool:
        return list(self) == list(other)

    def __repr__(self) -> str:
        return repr(list(self))


@dataclass
class ModelConfig:
    """ModelConfig (src/model/types.zig:43-62); layer_types default every 5th full (:109)."""
    vocab_size: int = 262144
    hidden_size: int = 1536
    intermediate_size: int = 12288
    num_hidden_layers: int = 35
    num_attention_heads: int = 8
    num_key_value_heads: int = 1
    head_dim: int = 256
    rotary_dim: int = 256
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    rope_theta_full: float = 1000000.0
    sliding_window: int = 512
    max_seq_len: int = 4096
    max_prefill_tokens: int = 1024
    layer_types: list = field(default_factory=list)  # True = full attention

    def __post_init__(self):
        if not self.layer_types:
            self.layer_types = [((l + 1) % 5 == 0) for l in range(self.num_hidden_layers)]

    @property
    def q_dim(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_key_value_heads * self.head_dim

    def to_c(self) -> L.ChModelConfig:
        c = L.ChModelConfig()
        for f in ("vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads",
                  "num_key_value_heads", "head_dim", "rotary_dim", "rms_norm_eps", "rope_theta", "rope_theta_full",
                  "sliding_window", "max_prefill_tokens"):
            setattr(c, f, getattr(self, f))
        for i, full in enumerate(self.layer_types[:64]):
            c.layer_types[i] = 1 if full else 0
        return c


def config_12b(layers: int = 48) -> ModelConfig:
    """12B-shape Q4 decoder (sliding window 1024 so decode and
    batched prefill agree, batch_causal_attn.wgsl:53)."""
    return ModelConfig(vocab_size=262144, hidden_size=3840, intermediate_size=15360, num_hidden_layers=layers,
                       num_attention_heads=16, num_key_value_heads=8, head_dim=256, rotary_dim=256,
                       sliding_window=1024)


class GpuContext:
    """GpuContext (src/gpu/context.zig): one CUDA device + one stream."""

    def __init__(self, handle: int, device: int):
        self.handle = handle
        self.device = device

    @classmethod
    def init(cls, device: int = 0) -> "GpuContext":
        lib = L.load()
        h = C.c_void_p()
        L.check(lib.ch_ctx_create(device, C.byref(h)))
        return cls(h.value, device)

    def deinit(self) -> None:
        if self.handle:
            L.load().ch_ctx_destroy(self.handle)
            self.handle = None

    def synchronize(self) -> None:
        L.check(L.load().ch_ctx_synchronize(self.handle))

    @property
    def stream(self) -> int:
        return L.load().ch_ctx_stream(self.handle)

    def device_status(self) -> int:
        f = C.c_uint32()
        L.check(L.load().ch_ctx_device_status(self.handle, C.byref(f)))
        return f.value


@dataclass
class LayerWeightsQ4:
    """LayerWeights (src/model/types.zig:13-41) with projections already in
    quantizeRowQ4_0 block form (uint32 [rows, cols/32*5]) and f32 norms."""
    q_proj: np.ndarray
    k_proj: np.ndarray
    v_proj: np.ndarray
    o_proj: np.ndarray
    gate_proj: np.ndarray
    up_proj: np.ndarray
    down_proj: np.ndarray
    input_norm: np.ndarray
    q_norm: np.ndarray
    k_norm: np.ndarray
    pre_ffn_norm: np.ndarray
    post_attn_norm: Optional[np.ndarray] = None
    post_ffn_norm: Optional[np.ndarray] = None
    layer_scalar: float = 1.0


class GpuModelContext:
    """GpuModelContext (src/gpu/model_gpu.zig:30-216): device weights, KV, graphs."""

    def __init__(self, ctx: GpuContext, handle: int, config: ModelConfig):
        self.ctx = ctx
        self.handle = handle
        self.config = config

    @classmethod
    def init(cls, ctx: GpuContext, config: ModelConfig, layers: Sequence[LayerWeightsQ4], lm_head_q8: np.ndarray,
             final_norm: np.ndarray, embed_bf16: Optional[np.ndarray] = None) -> "GpuModelContext":
        lib = L.load()
        arr = (L.ChLayerWeights * len(layers))()
        keep = []
        for i, lw in enumerate(layers):
            w = arr[i]
            for name in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"):
                a = np.ascontiguousarray(getattr(lw, name), dtype=np.uint32)
                keep.append(a)
                setattr(w, name, _ptr(a, C.c_uint32))
            for name in ("input_norm", "q_norm", "k_norm", "pre_ffn_norm", "post_attn_norm", "post_ffn_norm"):
                v = getattr(lw, name)
                if v is None:
                    continue
                a = np.ascontiguousarray(v, dtype=np.float32)
                keep.append(a)
                setattr(w, name, _ptr(a, C.c_float))
            w.layer_scalar = lw.layer_scalar
        lm = np.ascontiguousarray(lm_head_q8, dtype=np.uint32)
        fn = np.ascontiguousarray(final_norm, dtype=np.float32)
        emb = None if embed_bf16 is None else np.ascontiguousarray(embed_bf16, dtype=np.uint16)
        cfg = config.to_c()
        h = C.c_void_p()
        L.check(lib.ch_model_create(ctx.handle, C.byref(cfg), arr, _ptr(lm, C.c_uint32), _ptr(fn, C.c_float),
                                    _ptr(emb, C.c_uint16), C.byref(h)))
        return cls(ctx, h.value, config)

    @classmethod
    def from_bf16(cls, ctx: GpuContext, config: ModelConfig, layers: Sequence[dict], embed_bf16: np.ndarray,
                  final_norm_bf16: Optional[np.ndarray] = None) -> "GpuModelContext":
        """GpuModelContext.init with quantize-on-load (src/gpu/model_gpu.zig:44-55,68-127):
        layers are dicts of bf16 (uint16) arrays named like LayerWeights (q_proj ...
        down_proj [out, in]; input_norm, q_norm, k_norm, pre_ffn_norm, post_attn_norm,
        post_ffn_norm; optional layer_scalar).  Missing v_proj = k_proj; missing norms
        follow ch_model_create_bf16."""
        lib = L.load()
        arr = (L.ChLayerWeightsBf16 * len(layers))()
        keep = []
        for i, lw in enumerate(layers):
            w = arr[i]
            for name in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj", "input_norm",
                         "q_norm", "k_norm", "post_attn_norm", "pre_ffn_norm", "post_ffn_norm"):
                v = lw.get(name)
                if v is None:
                    continue
                a = np.ascontiguousarray(v, dtype=np.uint16)
                keep.append(a)
                setattr(w, name, _ptr(a, C.c_uint16))
            w.layer_scalar = float(lw.get("layer_scalar", 1.0))
        emb = np.ascontiguousarray(embed_bf16, dtype=np.uint16)
        fn = None if final_norm_bf16 is None else np.ascontiguousarray(final_norm_bf16, dtype=np.uint16)
        cfg = config.to_c()
        h = C.c_void_p()
        L.check(lib.ch_model_create_bf16(ctx.handle, C.byref(cfg), arr, _ptr(emb, C.c_uint16), _ptr(fn, C.c_uint16),
                                         C.byref(h)))
        return cls(ctx, h.value, config)

    @classmethod
    def synthetic(cls, ctx: GpuContext, config: ModelConfig, seed: int) -> "GpuModelContext":
        lib = L.load()
        cfg = config.to_c()
        h = C.c_void_p()
        L.check(lib.ch_model_create_synthetic(ctx.handle, C.byref(cfg), seed, C.byref(h)))
        return cls(ctx, h.value, config)

    @classmethod
    def synthetic_sharded(cls, ctx: GpuContext, config: ModelConfig, seed: int, rank: int,
                          world: int) -> "GpuModelContext":
        """Shard `rank` of a `world`-GPU tensor-parallel model with the same synthetic
        weights as synthetic(); call attach_peers before decoding."""
        lib = L.load()
        cfg = config.to_c()
        h = C.c_void_p()
        L.check(lib.ch_model_create_synthetic_sharded(ctx.handle, C.byref(cfg), seed, rank, world, C.byref(h)))
        m = cls(ctx, h.value, config)
        m.rank, m.world = rank, world
        return m

    def exchange_handle(self) -> bytes:
        """CUDA IPC handle of this rank's exchange arena (CH_IPC_HANDLE_BYTES bytes)."""
        buf = (C.c_uint8 * L.CH_IPC_HANDLE_BYTES)()
        L.check(L.load().ch_model_exchange_handle(self.handle, buf))
        return bytes(buf)

    def attach_peers(self, handles: Sequence[bytes]) -> None:
        """Map every rank's arena; `handles` in rank order (this rank's included)."""
        blob = b"".join(handles)
        assert len(blob) == L.CH_IPC_HANDLE_BYTES * len(handles)
        buf = (C.c_uint8 * len(blob)).from_buffer_copy(blob)
        L.check(L.load().ch_model_attach_peers(self.handle, buf))

    def deinit(self) -> None:
        if self.handle:
            L.load().ch_model_destroy(self.handle)
            self.handle = None

    def zero_state(self) -> None:
        L.check(L.load().ch_model_zero_state(self.handle))

    def read_x(self) -> np.ndarray:
        x = np.empty(self.config.hidden_size, np.float32)
        L.check(L.load().ch_read_x(self.handle, _ptr(x, C.c_float)))
        return x

    def read_normed_x(self) -> np.ndarray:
        x = np.empty(self.config.hidden_size, np.float32)
        L.check(L.load().ch_read_normed_x(self.handle, _ptr(x, C.c_float)))
        return x

    def kv_read(self, layer: int, slot: int):
        k = np.empty(self.config.kv_dim, np.float32)
        v = np.empty(self.config.kv_dim, np.float32)
        L.check(L.load().ch_kv_read(self.handle, layer, slot, _ptr(k, C.c_float), _ptr(v, C.c_float)))
        return k, v

    def kv_write(self, layer: int, slot: int, k: np.ndarray, v: np.ndarray) -> None:
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        L.check(L.load().ch_kv_write(self.handle, layer, slot, _ptr(k, C.c_float), _ptr(v, C.c_float)))

    # device-resident greedy loop -------------------------------------------------
    def decode_plan(self, steps: Sequence[tuple]) -> None:
        """steps: (clock, slot, active_list, sliding_list) per step."""
        lib = L.load()
        arr = (L.ChStepDesc * len(steps))()
        keep = []
        for i, (clock, slot, act, sli) in enumerate(steps):
            a = np.ascontiguousarray(act, np.uint32)
            s = np.ascontiguousarray(sli, np.uint32)
            keep += [a, s]
            arr[i].clock, arr[i].slot, arr[i].n_active, arr[i].n_sliding = clock, slot, len(a), len(s)
            arr[i].active, arr[i].sliding = _ptr(a, C.c_uint32), _ptr(s, C.c_uint32)
        L.check(lib.ch_decode_plan(self.handle, arr, len(steps)))

    # ---- multi-stream greedy decode ----
    def streams_init(self, n_streams: int, max_batch: int) -> None:
        """Per-stream 4,096-slot KV caches for n_streams; steps of up to max_batch streams."""
        L.check(L.load().ch_streams_init(self.handle, n_streams, max_batch))

    def stream_prefill(self, stream: int, tokens, slots, start_clock: int, num_prev: int) -> int:
        """Batched prefill of one stream's prompt into its own cache; returns the greedy next token."""
        t = np.ascontiguousarray(tokens, np.uint32)
        sl = np.ascontiguousarray(slots, np.uint32)
        out = C.c_uint32()
        L.check(L.load().ch_stream_prefill(self.handle, stream, _ptr(t, C.c_uint32), len(t), _ptr(sl, C.c_uint32),
                                           start_clock, num_prev, C.byref(out)))
        return int(out.value)

    def streams_decode(self, steps: Sequence[tuple]) -> np.ndarray:
        """One batched step; steps: (stream, token, clock, slot, active_list, sliding_list).
        Returns each stream's greedy next token (step order)."""
        arr = (L.ChStreamStep * len(steps))()
        keep = []
        for i, (stream, token, clock, slot, act, sli) in enumerate(steps):
            a = np.ascontiguousarray(act, np.uint32)
            s = np.ascontiguousarray(sli, np.uint32)
            keep += [a, s]
            arr[i].stream, arr[i].token, arr[i].clock, arr[i].slot = stream, token, clock, slot
            arr[i].active, arr[i].sliding = _ptr(a, C.c_uint32), _ptr(s, C.c_uint32)
            arr[i].n_active, arr[i].n_sliding = len(a), len(s)
        out = np.zeros(len(steps), np.uint32)
        L.check(L.load().ch_streams_decode(self.handle, arr, len(steps), _ptr(out, C.c_uint32)))
        return out

    def streams_read_normed_x(self, n: int) -> np.ndarray:
        """final-normed hidden state of each of the last streams step's n tokens"""
        out = np.empty((n, self.config.hidden_size), np.float32)
        L.check(L.load().ch_streams_read_normed_x(self.handle, n, _ptr(out, C.c_float)))
        return out

    def streams_read_logits(self, n: int) -> np.ndarray:
        """raw (pre-softcap) logits of each of the last streams step's n tokens"""
        out = np.empty((n, self.config.vocab_size), np.float32)
        L.check(L.load().ch_streams_read_logits(self.handle, n, _ptr(out, C.c_float)))
        return out

    def streams_decode_steps(self, steps, n: int) -> np.ndarray:
        """One batched step from n prepared ChStreamStep records (ch_rings_fill_steps)."""
        out = np.zeros(n, np.uint32)
        L.check(L.load().ch_streams_decode(self.handle, steps, n, _ptr(out, C.c_uint32)))
        return out

    def decode_run(self, first_token: int, n_steps: int) -> None:
        L.check(L.load().ch_decode_run(self.handle, first_token, n_steps))

    def decode_continue(self, n_steps: int) -> None:
        L.check(L.load().ch_decode_continue(self.handle, n_steps))

    def weight_tiles(self, layer: int, which: int):
        """(device pointer, rows, cols) of a repacked weight: 0 qkv, 1 o, 2 gate|up, 3 down, 4 LM head."""
        ptr, rows, cols = C.c_void_p(), C.c_uint32(), C.c_uint32()
        L.check(L.load().ch_model_weight_tiles(self.handle, layer, which, C.byref(ptr), C.byref(rows), C.byref(cols)))
        return ptr.value, rows.value, cols.value

    def decode_tokens(self, n: int) -> np.ndarray:
        t = np.empty(n, np.uint32)
        L.check(L.load().ch_decode_tokens(self.handle, _ptr(t, C.c_uint32), n))
        return t

    def decode_run_ring(self, ring_dev: "DeviceRing", host_ring: Optional["DynamicRingBuffer"], first_token: int,
                        first_clock: int, n_steps: int) -> None:
        """device-resident loop whose ring lists are built on the device (ch_decode_run_ring)"""
        L.check(L.load().ch_decode_run_ring(self.handle, ring_dev.h, host_ring.h if host_ring else None, first_token,
                                            first_clock, n_steps))

    def set_sampler(self, sampler: Optional["DeviceSampler"]) -> None:
        """device loops sample with `sampler` (Sampler.sampleTopK on the device); None = greedy"""
        L.check(L.load().ch_model_set_sampler(self.handle, sampler.h if sampler else None))


class DeviceRing:
    """device copy of a ring's layer-0 slot metadata (ch_ring_dev_*)"""

    def __init__(self, ctx: GpuContext):
        h = C.c_void_p()
        L.check(L.load().ch_ring_dev_create(ctx.handle, C.byref(h)))
        self.h = h.value

    def upload(self, ring: "DynamicRingBuffer") -> None:
        L.check(L.load().ch_ring_dev_upload(self.h, ring.h))

    def deinit(self) -> None:
        if self.h:
            L.load().ch_ring_dev_destroy(self.h)
            self.h = None


class DeviceSampler:
    """Sampler (src/sampler.zig:55-82) whose sampleTopK runs on the device (ch_sampler_*)"""

    def __init__(self, ctx: GpuContext, seed: int, temp: float, top_p: float, min_p: float = 0.05,
                 repeat_penalty: float = 1.1, frequency_penalty: float = 0.1, presence_penalty: float = 0.1,
                 suppress_thinking: bool = False, suppress_critique: bool = False,
                 suppress_channel_close: bool = False, recent_cap: int = 8192):
        p = L.ChSamplerParams(temp, top_p, min_p, repeat_penalty, frequency_penalty, presence_penalty, 64,
                              int(suppress_thinking), int(suppress_critique), int(suppress_channel_close), 0)
        h = C.c_void_p()
        L.check(L.load().ch_sampler_create(ctx.handle, C.byref(p), seed, recent_cap, C.byref(h)))
        self.h = h.value

    def set_recent(self, tokens: Sequence[int]) -> None:
        t = np.ascontiguousarray(tokens, np.uint32)
        L.check(L.load().ch_sampler_set_recent(self.h, _ptr(t, C.c_uint32), t.size))

    def deinit(self) -> None:
        if self.h:
            L.load().ch_sampler_destroy(self.h)
            self.h = None


def gpu_dispatch_forward_token(gpu: GpuModelContext, x: np.ndarray, clock: int, slot_idx: int,
                               active_slots: Sequence[int], sliding_slots: Sequence[int],
                               topk_out: bool = True) -> tuple[int, Optional[list]]:
    """gpuDispatchForwardToken (src/gpu/model_dispatch.zig:128-153).

    Returns (greedy token, the 64 TopKCandidate as a sequence, or None)."""
    lib = L.load()
    x = np.ascontiguousarray(x, np.float32)
    act = np.ascontiguousarray(active_slots, np.uint32)
    sli = np.ascontiguousarray(sliding_slots, np.uint32)
    tk = (L.ChTopk * 64)() if topk_out else None
    tok = C.c_uint32(0)
    L.check(lib.ch_forward_token(gpu.handle, _ptr(x, C.c_float), clock, slot_idx, _ptr(act, C.c_uint32), len(act),
                                 _ptr(sli, C.c_uint32), len(sli), tk, C.byref(tok) if topk_out else None))
    return tok.value, (TopKList(tk) if topk_out else None)


def gpu_dispatch_prefill_batch(gpu: GpuModelContext, tokens: Sequence[int], embed_tokens: Optional[np.ndarray],
                               slots: Sequence[int], start_clock: int, num_prev_slots: int, want_topk: bool = True,
                               progress_fn: Optional[Callable[[int, int], None]] = None,
                               logits_out: Optional[np.ndarray] = None) -> Optional[list]:
    """gpuDispatchPrefillBatch (src/gpu/batch_dispatch.zig:27-172).  embed_tokens is
    the bf16 table as uint16 (None = the model's device table); logits_out, a float32
    array of at most vocab entries, receives the last token's raw logits
    (batch_dispatch.zig:168-170)."""
    lib = L.load()
    tok = np.ascontiguousarray(tokens, np.uint32)
    sl = np.ascontiguousarray(slots, np.uint32)
    emb = None if embed_tokens is None else np.ascontiguousarray(embed_tokens, np.uint16)
    tk = (L.ChTopk * 64)() if want_topk else None
    cb = L.PROGRESS_FN(lambda i, n, _c: progress_fn(i, n)) if progress_fn else L.PROGRESS_FN()
    if logits_out is not None:
        assert logits_out.dtype == np.float32 and logits_out.flags.c_contiguous
    L.check(lib.ch_prefill(gpu.handle, _ptr(tok, C.c_uint32), len(tok), _ptr(emb, C.c_uint16), _ptr(sl, C.c_uint32),
                           start_clock, num_prev_slots, tk, _ptr(logits_out, C.c_float),
                           0 if logits_out is None else logits_out.size, cb, None))
    return [TopKCandidate(t.id, t.val) for t in tk] if want_topk else None


class DynamicRingBuffer:
    """DynamicRingBuffer slot math (src/ring_buffer.zig:21-391) backed by the C++ ring."""

    def __init__(self, num_layers: int, num_anchors: int = 0):
        self._lib = L.load()
        self.h = self._lib.ch_ring_create(num_layers, num_anchors)
        self.num_layers = num_layers

    def deinit(self) -> None:
        if self.h:
            self._lib.ch_ring_destroy(self.h)
            self.h = None

    def reset(self):
        self._lib.ch_ring_reset(self.h)

    def setNumAnchors(self, n: int):
        self._lib.ch_ring_set_num_anchors(self.h, n)

    @property
    def num_anchors(self) -> int:
        return self._lib.ch_ring_num_anchors(self.h)

    @property
    def total_ingested(self) -> int:
        return self._lib.ch_ring_total_ingested(self.h)

    def windowSize(self, layer: int = 0) -> int:
        return self._lib.ch_ring_window_size(self.h, layer)

    def getSlotIndex(self, clock: int) -> int:
        return self._lib.ch_ring_get_slot_index(self.h, 0, clock)

    def getSlotIndexLayer(self, layer: int, clock: int) -> int:
        return self._lib.ch_ring_get_slot_index(self.h, layer, clock)

    def activateSlot(self, layer: int, clock: int) -> int:
        return self._lib.ch_ring_activate_slot(self.h, layer, clock)

    def activateRange(self, clock0: int, n: int) -> np.ndarray:
        """activateSlot of clocks [clock0, clock0 + n) in every layer; returns their slots."""
        out = np.empty(n, np.uint32)
        self._lib.ch_ring_activate_range(self.h, clock0, n, _ptr(out, C.c_uint32))
        return out

    def deactivateSlot(self, layer: int, clock: int):
        self._lib.ch_ring_deactivate_slot(self.h, layer, clock)

    def rollbackClock(self, target: int):
        self._lib.ch_ring_rollback_clock(self.h, target)

    def writeKV(self, layer: int, clock: int):
        """Metadata half of writeKV; the K/V rows are written by the kernels."""
        self._lib.ch_ring_write_kv_meta(self.h, layer, clock)

    def writeRecallKV(self, layer: int, rank: int, clock: int):
        self._lib.ch_ring_write_recall_meta(self.h, layer, rank, clock)

    def clearRecall(self):
        self._lib.ch_ring_clear_recall(self.h)

    def markBoundary(self, clock: int, span_type: int = 6, salience: float = 1.0):
        self._lib.ch_ring_mark_boundary(self.h, clock, span_type, salience)

    def is_active(self, layer: int, slot: int) -> bool:
        return bool(self._lib.ch_ring_is_active(self.h, layer, slot))

    def slot_clock(self, layer: int, slot: int) -> int:
        return self._lib.ch_ring_slot_clock(self.h, layer, slot)

    def getActiveSlotsLayer(self, layer: int, clock: int, is_sliding: bool, sliding_window: int) -> np.ndarray:
        if getattr(self, "_out", None) is None:  # one output buffer per ring, reused by every call
            self._out = np.empty(TOTAL_SLOTS, np.uint32)
            self._out_p = _ptr(self._out, C.c_uint32)
        n = self._lib.ch_ring_active_slots(self.h, layer, clock, 1 if is_sliding else 0, sliding_window, self._out_p)
        return self._out[:n].copy()

    def getActiveSlots(self, layer: int, clock: int) -> np.ndarray:
        return self.getActiveSlotsLayer(layer, clock, False, 1024)

    def getPrefillPrevSlots(self, layer: int, start_clock: int, chunk_len: int) -> np.ndarray:
        out = np.empty(TOTAL_SLOTS, np.uint32)
        n = self._lib.ch_ring_prefill_prev_slots(self.h, layer, start_clock, chunk_len, _ptr(out, C.c_uint32))
        return out[:n].copy()


def attach_tensor_parallel(gm: "GpuModelContext", group=None) -> None:
    """All-gather the ranks' arena handles over torch.distributed (any backend:
    gloo on the host or NCCL) and attach them -- the only host-side exchange a
    tensor-parallel model needs."""
    import torch
    import torch.distributed as dist

    mine = torch.tensor(list(gm.exchange_handle()), dtype=torch.uint8)
    backend = dist.get_backend(group)
    if backend == "nccl":
        mine = mine.cuda()
    world = dist.get_world_size(group)
    parts = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(parts, mine, group=group)
    gm.attach_peers([bytes(p.cpu().tolist()) for p in parts])
