"""ctypes wrapper of liboracle.so -- the CPU restatement of the reference hot path.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / --impl reference leg, never by the product package.
Parity status is documented in channel_oracle.h (ring/sampler/bf16 pinned by
the reference's own known-answer tests; matvec/attention/norm/RoPE restated
from the reference sources, "parity unpinned" by any reference-run vector).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"

u8, u16, u32, u64, f32, sz, i32 = C.c_uint8, C.c_uint16, C.c_uint32, C.c_uint64, C.c_float, C.c_size_t, C.c_int
vp = C.c_void_p
P = C.POINTER

# tensor ids of the seeded generator (identical to channel_b200/csrc/model.cu)
T_Q, T_K, T_V, T_O, T_GATE, T_UP, T_DOWN = 0, 1, 2, 3, 4, 5, 6
T_IN_NORM, T_Q_NORM, T_K_NORM, T_POST_ATTN, T_PRE_FFN, T_POST_FFN = 10, 11, 12, 13, 14, 15
T_EMBED, T_FINAL_NORM = 20, 21
WEIGHT_STD = 0.02


class OrModelCfg(C.Structure):
    _fields_ = [("vocab", u32), ("hidden", u32), ("inter", u32), ("layers", u32), ("n_q", u32), ("n_kv", u32),
                ("head_dim", u32), ("rot_dim", u32), ("eps", f32), ("theta_sliding", f32), ("theta_full", f32),
                ("sliding_window", u32), ("layer_full", u8 * 64)]


class OrLayer(C.Structure):
    _fields_ = [("wq", P(u32)), ("wk", P(u32)), ("wv", P(u32)), ("wo", P(u32)), ("wg", P(u32)), ("wu", P(u32)),
                ("wd", P(u32)), ("input_norm", P(f32)), ("q_norm", P(f32)), ("k_norm", P(f32)),
                ("post_attn_norm", P(f32)), ("pre_ffn_norm", P(f32)), ("post_ffn_norm", P(f32)),
                ("layer_scalar", f32)]


_SIG = {
    "or_bf16_from_f32": (u16, [f32]), "or_bf16_to_f32": (f32, [u16]),
    "or_f16_from_f32": (u16, [f32]), "or_f16_to_f32": (f32, [u16]),
    "or_quantize_row_q4": (None, [P(u32), P(u16), sz]), "or_quantize_row_q8": (None, [P(u32), P(u16), sz]),
    "or_quantize_matrix": (None, [P(u32), P(u16), sz, sz, i32, i32]),
    "or_tensor_seed": (u64, [u64, u32, u32]), "or_gen_normal": (f32, [u64, u64, u64]),
    "or_gen_q4_matrix": (None, [P(u32), sz, sz, u64, f32, i32]),
    "or_gen_bf16": (None, [P(u16), sz, u64, f32, f32, i32]), "or_gen_f32": (None, [P(f32), sz, u64, f32, f32]),
    "or_gemv_q4": (None, [P(f32), P(u32), P(f32), sz, sz, i32]),
    "or_gemv_q8": (None, [P(f32), P(u32), P(f32), sz, sz, i32]),
    "or_fused_mlp_q4": (None, [P(f32), P(u32), P(u32), P(f32), sz, sz, i32]),
    "or_gelu_tanh": (f32, [f32]),
    "or_rmsnorm": (None, [P(f32), P(f32), P(f32), sz, f32]),
    "or_add_rmsnorm": (None, [P(f32), P(f32), P(f32), P(f32), sz, f32, f32]),
    "or_rope_inv_freq": (None, [P(f32), u32, f32]),
    "or_qkv_rope": (None, [P(f32), P(u16), P(u16), P(f32), P(f32), P(f32), P(f32), P(f32), u32, u32, u32, u32, i32,
                           f32, f32, u32, u32]),
    "or_decode_attn": (None, [P(f32), P(f32), P(u16), P(u16), P(u32), u32, u32, u32, u32, f32]),
    "or_topk64": (None, [P(u32), P(f32), P(f32), sz]), "or_argmax": (u32, [P(f32), sz]), "or_softcap": (f32, [f32]),
    "or_sample_topk_greedy": (u32, [P(u32), P(f32), sz, P(u32), sz, f32, f32, f32, i32, i32, i32]),
    "or_prng_seed": (None, [P(u64), u64]), "or_prng_next": (u64, [P(u64)]), "or_prng_float": (f32, [P(u64)]),
    "or_sample_topk": (u32, [P(u32), P(f32), sz, P(u32), sz, P(f32), i32, P(u64)]),
    "or_batch_gemm_q4": (None, [P(f32), P(u32), P(f32), sz, sz, sz, i32]),
    "or_batch_fused_mlp_q4": (None, [P(f32), P(u32), P(u32), P(f32), sz, sz, sz, i32]),
    "or_batch_rmsnorm": (None, [P(f32), P(f32), P(f32), sz, sz, f32]),
    "or_batch_add_rmsnorm": (None, [P(f32), P(f32), P(f32), P(f32), sz, sz, f32, f32]),
    "or_batch_qkv_rope": (None, [P(f32), P(u16), P(u16), P(f32), P(f32), P(f32), P(f32), P(f32), u32, u32, u32, u32,
                                 u32, i32, f32, f32, u32, P(u32), u32]),
    "or_batch_causal_attn": (None, [P(f32), P(f32), P(u16), P(u16), P(u32), u32, u32, u32, u32, u32, f32, i32, i32]),
    "or_ring_create": (vp, [u32, u32]), "or_ring_destroy": (None, [vp]), "or_ring_reset": (None, [vp]),
    "or_ring_set_num_anchors": (None, [vp, sz]), "or_ring_num_anchors": (sz, [vp]),
    "or_ring_total_ingested": (sz, [vp]), "or_ring_window_size": (sz, [vp, sz]),
    "or_ring_recall_start": (sz, [vp, sz]), "or_ring_get_slot_index": (sz, [vp, sz, sz]),
    "or_ring_activate_slot": (sz, [vp, sz, sz]), "or_ring_deactivate_slot": (None, [vp, sz, sz]),
    "or_ring_rollback_clock": (None, [vp, sz]), "or_ring_write_kv_meta": (None, [vp, sz, sz]),
    "or_ring_write_recall_meta": (None, [vp, sz, sz, sz]), "or_ring_clear_recall": (None, [vp]),
    "or_ring_mark_boundary": (None, [vp, sz, i32, f32]), "or_ring_record_attention": (None, [vp, sz, sz, f32]),
    "or_ring_attention_mass": (f32, [vp, sz, sz]), "or_ring_slot_salience": (f32, [vp, sz]),
    "or_ring_working_set_gini": (f32, [vp]), "or_ring_is_saturated": (i32, [vp, f32, f32]),
    "or_ring_evict_low_salience": (sz, [vp, sz, sz, sz]), "or_ring_is_active": (i32, [vp, sz, sz]),
    "or_ring_slot_clock": (sz, [vp, sz, sz]),
    "or_ring_active_slots": (sz, [vp, sz, sz, i32, sz, P(u32)]),
    "or_ring_prefill_prev_slots": (sz, [vp, sz, sz, sz, P(u32)]),
    "or_model_create": (vp, [P(OrModelCfg), P(OrLayer), P(u32), P(f32), i32]),
    "or_model_destroy": (None, [vp]), "or_model_reset_kv": (None, [vp]),
    "or_model_forward_token": (u32, [vp, P(f32), u32, u32, P(u32), u32, P(u32), u32, P(u32), P(f32)]),
    "or_model_prefill": (u32, [vp, P(f32), u32, P(u32), u32, u32, P(u32), P(f32)]),
    "or_model_x": (P(f32), [vp]), "or_model_normed_x": (P(f32), [vp]),
    "or_model_k_cache": (P(u16), [vp, u32]), "or_model_v_cache": (P(u16), [vp, u32]),
    "or_embed": (None, [P(f32), P(u16), P(u32), sz, sz]),
}

_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
        l = C.CDLL(str(LIB))
        for n, (r, a) in _SIG.items():
            fn = getattr(l, n)
            fn.restype, fn.argtypes = r, a
        _lib = l
    return _lib


def nthreads() -> int:
    return max(1, len(os.sched_getaffinity(0)))


def p(a, ct):
    return None if a is None else a.ctypes.data_as(P(ct))


# ---- generators ---------------------------------------------------------------
def tensor_seed(seed: int, layer: int, tid: int) -> int:
    return lib().or_tensor_seed(seed, layer, tid)


def gen_q4(rows: int, cols: int, tseed: int, std: float = WEIGHT_STD) -> np.ndarray:
    out = np.empty((rows, cols // 32 * 5), np.uint32)
    lib().or_gen_q4_matrix(p(out, u32), rows, cols, tseed, std, nthreads())
    return out


def gen_bf16(n: int, tseed: int, mean: float, std: float) -> np.ndarray:
    out = np.empty(n, np.uint16)
    lib().or_gen_bf16(p(out, u16), n, tseed, mean, std, nthreads())
    return out


def gen_f32(n: int, tseed: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().or_gen_f32(p(out, f32), n, tseed, mean, std)
    return out


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


def quantize_matrix(src_bf16: np.ndarray, rows: int, cols: int, mode: int) -> np.ndarray:
    out = np.empty((rows, cols // 32 * (9 if mode == 8 else 5)), np.uint32)
    src = np.ascontiguousarray(src_bf16, np.uint16)
    lib().or_quantize_matrix(p(out, u32), p(src, u16), rows, cols, mode, nthreads())
    return out


# ---- ops ------------------------------------------------------------------------
def gemv_q4(W: np.ndarray, x: np.ndarray, M: int, K: int) -> np.ndarray:
    y = np.empty(M, np.float32)
    lib().or_gemv_q4(p(y, f32), p(W, u32), p(np.ascontiguousarray(x, np.float32), f32), M, K, nthreads())
    return y


def gemv_q8(W: np.ndarray, x: np.ndarray, M: int, K: int) -> np.ndarray:
    y = np.empty(M, np.float32)
    lib().or_gemv_q8(p(y, f32), p(W, u32), p(np.ascontiguousarray(x, np.float32), f32), M, K, nthreads())
    return y


def fused_mlp_q4(Wg, Wu, x, M, K) -> np.ndarray:
    y = np.empty(M, np.float32)
    lib().or_fused_mlp_q4(p(y, f32), p(Wg, u32), p(Wu, u32), p(np.ascontiguousarray(x, np.float32), f32), M, K,
                          nthreads())
    return y


def topk64(logits: np.ndarray):
    ids = np.empty(64, np.uint32)
    vals = np.empty(64, np.float32)
    lg = np.ascontiguousarray(logits, np.float32)
    lib().or_topk64(p(ids, u32), p(vals, f32), p(lg, f32), lg.size)
    return ids, vals


def qkv_rope(q, k, v, q_norm, k_norm, k_cache, v_cache, nq, nkv, D, rot, theta, eps, clock, slot):
    q_out = np.empty(nq * D, np.float32)
    lib().or_qkv_rope(p(q_out, f32), p(k_cache, u16), p(v_cache, u16), p(q, f32), p(k, f32), p(v, f32),
                      p(q_norm, f32), p(k_norm, f32), nq, nkv, D, rot, 0, theta, eps, clock, slot)
    return q_out


def decode_attn(q, k_cache, v_cache, slots, nq, nkv, D, scale):
    out = np.empty(nq * D, np.float32)
    sl = np.ascontiguousarray(slots, np.uint32)
    lib().or_decode_attn(p(out, f32), p(q, f32), p(k_cache, u16), p(v_cache, u16), p(sl, u32), sl.size, nq, nkv, D,
                         scale)
    return out


def batch_causal_attn(Q, k_cache, v_cache, slots, N, num_prev, nq, nkv, D, scale, is_sliding) -> np.ndarray:
    """batch_causal_attn.wgsl:25-223: Q [N][nq*D] -> out [N][nq*D]"""
    out = np.empty((N, nq * D), np.float32)
    sl = np.ascontiguousarray(slots, np.uint32)
    lib().or_batch_causal_attn(p(out, f32), p(np.ascontiguousarray(Q, np.float32), f32), p(k_cache, u16),
                               p(v_cache, u16), p(sl, u32), N, num_prev, nq, nkv, D, scale, int(is_sliding), nthreads())
    return out


def batch_gemm_q4(W, X, N, M, K) -> np.ndarray:
    Y = np.empty((N, M), np.float32)
    lib().or_batch_gemm_q4(p(Y, f32), p(W, u32), p(np.ascontiguousarray(X, np.float32), f32), N, M, K, nthreads())
    return Y


def batch_fused_mlp_q4(Wg, Wu, X, N, M, K) -> np.ndarray:
    Y = np.empty((N, M), np.float32)
    lib().or_batch_fused_mlp_q4(p(Y, f32), p(Wg, u32), p(Wu, u32), p(np.ascontiguousarray(X, np.float32), f32), N, M,
                                K, nthreads())
    return Y


# ---- ring -----------------------------------------------------------------------
class Ring:
    """DynamicRingBuffer restatement (src/ring_buffer.zig), metadata only."""

    def __init__(self, num_layers: int, num_anchors: int):
        self.l = lib()
        self.h = self.l.or_ring_create(num_layers, num_anchors)

    def __del__(self):
        if getattr(self, "h", None):
            self.l.or_ring_destroy(self.h)
            self.h = None

    def __getattr__(self, name):
        fn = getattr(self.l, "or_ring_" + name)
        return lambda *a: fn(self.h, *a)

    def active_list(self, layer, clock, is_sliding, window) -> np.ndarray:
        out = np.empty(4096, np.uint32)
        n = self.l.or_ring_active_slots(self.h, layer, clock, int(is_sliding), window, p(out, u32))
        return out[:n].copy()

    def prefill_prev(self, layer, start_clock, chunk_len) -> np.ndarray:
        out = np.empty(4096, np.uint32)
        n = self.l.or_ring_prefill_prev_slots(self.h, layer, start_clock, chunk_len, p(out, u32))
        return out[:n].copy()


# ---- whole model ----------------------------------------------------------------
class SyntheticWeights:
    """Host copy of the seeded synthetic model (same tensors the CUDA generator makes)."""

    def __init__(self, cfg, seed: int, with_embed: bool = True):
        H, I, V = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size
        qd, kvd, D = cfg.q_dim, cfg.kv_dim, cfg.head_dim
        self.cfg = cfg
        self.layers = []
        ts = lambda l, t: tensor_seed(seed, l, t)  # noqa: E731
        for l in range(cfg.num_hidden_layers):
            norm = lambda n, t: bf16_to_f32(gen_bf16(n, ts(l, t), 1.0, 0.02))  # noqa: E731
            self.layers.append(dict(
                wq=gen_q4(qd, H, ts(l, T_Q)), wk=gen_q4(kvd, H, ts(l, T_K)), wv=gen_q4(kvd, H, ts(l, T_V)),
                wo=gen_q4(H, qd, ts(l, T_O)), wg=gen_q4(I, H, ts(l, T_GATE)), wu=gen_q4(I, H, ts(l, T_UP)),
                wd=gen_q4(H, I, ts(l, T_DOWN)),
                input_norm=norm(H, T_IN_NORM), q_norm=norm(D, T_Q_NORM), k_norm=norm(D, T_K_NORM),
                post_attn_norm=norm(H, T_POST_ATTN), pre_ffn_norm=norm(H, T_PRE_FFN), post_ffn_norm=norm(H, T_POST_FFN),
                layer_scalar=1.0))
        self.final_norm = bf16_to_f32(gen_bf16(H, ts(0, T_FINAL_NORM), 1.0, 0.02))
        self.embed = gen_bf16(V * H, ts(0, T_EMBED), 0.0, 0.02) if with_embed else None
        self.lm_head = quantize_matrix(self.embed, V, H, 8) if with_embed else None


class Model:
    """or_model: the reference's GPU-path layer order run on the CPU."""

    def __init__(self, cfg, w: SyntheticWeights):
        self.l = lib()
        c = OrModelCfg()
        c.vocab, c.hidden, c.inter, c.layers = cfg.vocab_size, cfg.hidden_size, cfg.intermediate_size, \
            cfg.num_hidden_layers
        c.n_q, c.n_kv, c.head_dim, c.rot_dim = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim, \
            cfg.rotary_dim
        c.eps, c.theta_sliding, c.theta_full = cfg.rms_norm_eps, cfg.rope_theta, cfg.rope_theta_full
        c.sliding_window = cfg.sliding_window
        for i, full in enumerate(cfg.layer_types[:64]):
            c.layer_full[i] = 1 if full else 0
        arr = (OrLayer * cfg.num_hidden_layers)()
        self._keep = [w]
        for i, lw in enumerate(w.layers):
            for k in ("wq", "wk", "wv", "wo", "wg", "wu", "wd"):
                setattr(arr[i], k, p(lw[k], u32))
            for k in ("input_norm", "q_norm", "k_norm", "post_attn_norm", "pre_ffn_norm", "post_ffn_norm"):
                if lw[k] is not None:
                    setattr(arr[i], k, p(lw[k], f32))
            arr[i].layer_scalar = lw["layer_scalar"]
        self._keep.append(arr)
        self.cfg = cfg
        self.h = self.l.or_model_create(C.byref(c), arr, p(w.lm_head, u32), p(w.final_norm, f32), nthreads())

    def __del__(self):
        if getattr(self, "h", None):
            self.l.or_model_destroy(self.h)
            self.h = None

    def forward_token(self, x, clock, slot, active, sliding):
        ids = np.empty(64, np.uint32)
        vals = np.empty(64, np.float32)
        a = np.ascontiguousarray(active, np.uint32)
        s = np.ascontiguousarray(sliding, np.uint32)
        tok = self.l.or_model_forward_token(self.h, p(np.ascontiguousarray(x, np.float32), f32), clock, slot, p(a, u32),
                                            a.size, p(s, u32), s.size, p(ids, u32), p(vals, f32))
        return tok, ids, vals

    def prefill(self, X, slots, start_clock, n_prev):
        ids = np.empty(64, np.uint32)
        vals = np.empty(64, np.float32)
        X = np.ascontiguousarray(X, np.float32)
        sl = np.ascontiguousarray(slots, np.uint32)
        tok = self.l.or_model_prefill(self.h, p(X, f32), X.shape[0], p(sl, u32), start_clock, n_prev, p(ids, u32),
                                      p(vals, f32))
        return tok, ids, vals

    def x(self) -> np.ndarray:
        return np.ctypeslib.as_array(self.l.or_model_x(self.h), shape=(self.cfg.hidden_size,)).copy()

    def normed_x(self) -> np.ndarray:
        return np.ctypeslib.as_array(self.l.or_model_normed_x(self.h), shape=(self.cfg.hidden_size,)).copy()

    def k_cache(self, layer) -> np.ndarray:
        return np.ctypeslib.as_array(self.l.or_model_k_cache(self.h, layer),
                                     shape=(4096 * self.cfg.kv_dim,)).copy()


def embed(table_bf16: np.ndarray, tokens, H: int) -> np.ndarray:
    tok = np.ascontiguousarray(tokens, np.uint32)
    out = np.empty((tok.size, H), np.float32)
    lib().or_embed(p(out, f32), p(np.ascontiguousarray(table_bf16, np.uint16), u16), p(tok, u32), tok.size, H)
    return out


# ---- sampler ----------------------------------------------------------------------
class Sampler:
    """Sampler.sampleTopK (src/sampler.zig:217-317) with Zig's DefaultPrng stream."""

    def __init__(self, seed: int, temp: float, top_p: float, min_p: float = 0.05, repeat_penalty: float = 1.1,
                 frequency_penalty: float = 0.1, presence_penalty: float = 0.1, suppress_thinking: bool = False,
                 suppress_critique: bool = False, suppress_channel_close: bool = False):
        self.state = np.zeros(4, np.uint64)
        lib().or_prng_seed(p(self.state, u64), seed)
        self.params = np.array([temp, top_p, min_p, repeat_penalty, frequency_penalty, presence_penalty], np.float32)
        self.flags = int(suppress_thinking) | (int(suppress_critique) << 1) | (int(suppress_channel_close) << 2)

    def sample_topk(self, ids, vals, recent=None) -> int:
        ids = np.ascontiguousarray(ids, np.uint32)
        vals = np.ascontiguousarray(vals, np.float32)
        rec = None if recent is None else np.ascontiguousarray(recent, np.uint32)
        return int(lib().or_sample_topk(p(ids, u32), p(vals, f32), ids.size, p(rec, u32),
                                        0 if rec is None else rec.size, p(self.params, f32), self.flags,
                                        p(self.state, u64)))

    def float32(self) -> float:
        return float(lib().or_prng_float(p(self.state, u64)))
