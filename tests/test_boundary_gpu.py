"""Drop-in boundary calls beyond forward_token / prefill's top-64, against the oracle:

* ch_prefill's logits_out -- gpuDispatchPrefillBatch copies the first
  logits_out.len raw logits of the last token (src/gpu/batch_dispatch.zig:36,168-170);
* ch_model_create_bf16 -- GpuModelContext.init quantizes bf16 weights on upload
  (src/gpu/model_gpu.zig:44-55,109-127,157); the model must decode exactly like the
  oracle built from quant.zig blocks of the same bf16 tensors;
* ch_kv_write / ch_kv_read -- the KV rows memory recall and snapshots write and read
  (src/memory.zig:99-121, src/snapshot.zig:95-98): a written row is read back as f16
  and attended to by the next decode step exactly like the oracle's cache row."""
import numpy as np
import pytest

from channel_b200 import DynamicRingBuffer, GpuModelContext, gpu_dispatch_forward_token, gpu_dispatch_prefill_batch
from channel_b200 import _lib as L
from tests.gpu_util import assert_close
from tests.model_util import ring_step_lists, small_config, topk_diff, topk_ids_agree

pytestmark = pytest.mark.gpu
SEED = 5


def _prompt_slots(ring, cfg, n):
    prev = ring.getPrefillPrevSlots(0, 0, n)
    slots = np.concatenate([prev, [ring.getSlotIndex(c) for c in range(n)]]).astype(np.uint32)
    for c in range(n):
        for layer in range(cfg.num_hidden_layers):
            ring.activateSlot(layer, c)
    return slots, len(prev)


def test_prefill_logits_out_matches_oracle(ctx, oracle):
    cfg = small_config()
    gm = GpuModelContext.synthetic(ctx, cfg, SEED)
    w = oracle.SyntheticWeights(cfg, SEED)
    om = oracle.Model(cfg, w)
    try:
        N = 24
        prompt = np.random.default_rng(3).integers(0, cfg.vocab_size, N).astype(np.uint32)
        ring = DynamicRingBuffer(cfg.num_hidden_layers, 0)
        slots, n_prev = _prompt_slots(ring, cfg, N)
        logits = np.full(cfg.vocab_size, np.nan, np.float32)
        cands = gpu_dispatch_prefill_batch(gm, prompt, None, slots, 0, n_prev, logits_out=logits)
        rtok, rid, rvals = om.prefill(oracle.embed(w.embed, prompt, cfg.hidden_size), slots, 0, n_prev)
        ref = oracle.gemv_q8(w.lm_head, om.normed_x(), cfg.vocab_size, cfg.hidden_size)
        assert_close(logits, ref, what="prefill logits_out vs oracle LM head")
        assert cands[0].id == rtok
        # the top-64 is the softcapped top of these very logits
        capped = 30.0 * np.tanh(logits.astype(np.float64) / 30.0)
        order = np.lexsort((np.arange(cfg.vocab_size), -capped))[:64]
        assert topk_ids_agree([c.id for c in cands], order, capped[order])
        # a shorter slice gets the prefix, and no top-64 is needed for it
        gm.zero_state()
        part = np.zeros(100, np.float32)
        ring2 = DynamicRingBuffer(cfg.num_hidden_layers, 0)
        slots2, n_prev2 = _prompt_slots(ring2, cfg, N)
        gpu_dispatch_prefill_batch(gm, prompt, None, slots2, 0, n_prev2, want_topk=False, logits_out=part)
        np.testing.assert_array_equal(part, logits[:100])
        # longer than the vocabulary: refused before any work
        with pytest.raises(L.ChannelError) as e:
            gpu_dispatch_prefill_batch(gm, prompt, None, slots2, 0, n_prev2,
                                       logits_out=np.zeros(cfg.vocab_size + 1, np.float32))
        assert e.value.status == L.CH_EINVAL
    finally:
        gm.deinit()


def _bf16(a: np.ndarray) -> np.ndarray:
    """f32 -> bf16 bits, round to nearest even (src/tensor.zig:7-13)"""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


class _Weights:
    """oracle-side weights built from the same bf16 tensors with quant.zig's quantizers"""

    def __init__(self, oracle, cfg, layers_bf16, embed, final_norm):
        H, I, qd, kvd = cfg.hidden_size, cfg.intermediate_size, cfg.q_dim, cfg.kv_dim
        shapes = {"q_proj": (qd, H), "k_proj": (kvd, H), "v_proj": (kvd, H), "o_proj": (H, qd),
                  "gate_proj": (I, H), "up_proj": (I, H), "down_proj": (H, I)}
        names = {"q_proj": "wq", "k_proj": "wk", "v_proj": "wv", "o_proj": "wo", "gate_proj": "wg",
                 "up_proj": "wu", "down_proj": "wd"}
        self.layers = []
        for lw in layers_bf16:
            d = {names[k]: oracle.quantize_matrix(lw[k], r, c, 4) for k, (r, c) in shapes.items()}
            for k in ("input_norm", "q_norm", "k_norm", "post_attn_norm", "pre_ffn_norm", "post_ffn_norm"):
                d[k] = oracle.bf16_to_f32(lw[k])
            d["layer_scalar"] = lw["layer_scalar"]
            self.layers.append(d)
        self.embed = embed
        self.final_norm = oracle.bf16_to_f32(final_norm)
        self.lm_head = oracle.quantize_matrix(embed, cfg.vocab_size, H, 8)


def test_bf16_model_quantized_on_load_matches_oracle(ctx, oracle):
    cfg = small_config()
    H, I, qd, kvd, D = cfg.hidden_size, cfg.intermediate_size, cfg.q_dim, cfg.kv_dim, cfg.head_dim
    rng = np.random.default_rng(21)
    mat = lambda r, c: _bf16(rng.standard_normal((r, c)).astype(np.float32) * 0.02)  # noqa: E731
    vec = lambda n: _bf16(1.0 + rng.standard_normal(n).astype(np.float32) * 0.02)  # noqa: E731
    layers = [dict(q_proj=mat(qd, H), k_proj=mat(kvd, H), v_proj=mat(kvd, H), o_proj=mat(H, qd), gate_proj=mat(I, H),
                   up_proj=mat(I, H), down_proj=mat(H, I), input_norm=vec(H), q_norm=vec(D), k_norm=vec(D),
                   post_attn_norm=vec(H), pre_ffn_norm=vec(H), post_ffn_norm=vec(H), layer_scalar=1.0)
              for _ in range(cfg.num_hidden_layers)]
    embed = mat(cfg.vocab_size, H)
    final_norm = vec(H)
    gm = GpuModelContext.from_bf16(ctx, cfg, layers, embed, final_norm)
    try:
        w = _Weights(oracle, cfg, layers, embed, final_norm)
        om = oracle.Model(cfg, w)
        N = 12
        prompt = rng.integers(0, cfg.vocab_size, N).astype(np.uint32)
        ring = DynamicRingBuffer(cfg.num_hidden_layers, 0)
        slots, n_prev = _prompt_slots(ring, cfg, N)
        cands = gpu_dispatch_prefill_batch(gm, prompt, None, slots, 0, n_prev)
        rtok, rid, rvals = om.prefill(oracle.embed(embed, prompt, H), slots, 0, n_prev)
        assert cands[0].id == rtok
        assert_close(gm.read_normed_x(), om.normed_x(), what="bf16 model: prefill normed x")
        tok = int(rtok)
        for clock in range(N, N + 5):
            slot, act, sli = ring_step_lists(ring, cfg, clock)
            x = oracle.embed(embed, [tok], H)[0]
            gtok, gc = gpu_dispatch_forward_token(gm, x, clock, slot, act, sli)
            r, rid, rvals = om.forward_token(x, clock, slot, act, sli)
            assert gtok == r, f"bf16 model: token at clock {clock}"
            # the prompt went through the tensor-core prefill (f32 sums not rounded like the
            # shader's, ~1e-4 relative on the hidden state), and logits of ~1 with cancelling
            # terms amplify that: ids are held exact away from near-ties at the 1e-3 float bar
            gi, gv = [c.id for c in gc], [c.val for c in gc]
            assert topk_ids_agree(gi, rid, rvals, tol=1e-3), f"clock {clock}: {topk_diff(gi, gv, rid, rvals)}"
            np.testing.assert_allclose(gv, rvals, rtol=1e-3, atol=1e-3)
            assert_close(gm.read_normed_x(), om.normed_x(), what=f"bf16 model: normed x at clock {clock}")
            tok = int(gtok)
    finally:
        gm.deinit()


def test_bf16_model_rejects_missing_weights(ctx):
    cfg = small_config()
    with pytest.raises(L.ChannelError) as e:
        GpuModelContext.from_bf16(ctx, cfg, [dict() for _ in range(cfg.num_hidden_layers)],
                                  np.zeros((cfg.vocab_size, cfg.hidden_size), np.uint16))
    assert e.value.status == L.CH_EINVAL
    assert b"q|k|v" in L.load().ch_last_error()


def test_kv_write_read_and_attend_like_oracle(ctx, oracle):
    cfg = small_config()
    gm = GpuModelContext.synthetic(ctx, cfg, SEED)
    w = oracle.SyntheticWeights(cfg, SEED)
    om = oracle.Model(cfg, w)
    try:
        gm.zero_state()
        ring = DynamicRingBuffer(cfg.num_hidden_layers, 0)
        rng = np.random.default_rng(9)
        tok = 11
        for clock in range(6):  # a few ordinary steps first
            slot, act, sli = ring_step_lists(ring, cfg, clock)
            x = oracle.embed(w.embed, [tok], cfg.hidden_size)[0]
            tok, _ = gpu_dispatch_forward_token(gm, x, clock, slot, act, sli)
            om.forward_token(x, clock, slot, act, sli)
        # memory recall: overwrite slots 2 and 4 of every layer on both sides
        for layer in range(cfg.num_hidden_layers):
            kc = np.ctypeslib.as_array(om.l.or_model_k_cache(om.h, layer), shape=(4096 * cfg.kv_dim,))
            vc = np.ctypeslib.as_array(om.l.or_model_v_cache(om.h, layer), shape=(4096 * cfg.kv_dim,))
            for s in (2, 4):
                k = rng.standard_normal(cfg.kv_dim).astype(np.float32)
                v = rng.standard_normal(cfg.kv_dim).astype(np.float32)
                gm.kv_write(layer, s, k, v)
                kh, vh = k.astype(np.float16), v.astype(np.float16)
                kc[s * cfg.kv_dim:(s + 1) * cfg.kv_dim] = kh.view(np.uint16)
                vc[s * cfg.kv_dim:(s + 1) * cfg.kv_dim] = vh.view(np.uint16)
                rk, rv = gm.kv_read(layer, s)
                np.testing.assert_array_equal(rk, kh.astype(np.float32))
                np.testing.assert_array_equal(rv, vh.astype(np.float32))
        for clock in range(6, 10):
            slot, act, sli = ring_step_lists(ring, cfg, clock)
            x = oracle.embed(w.embed, [int(tok)], cfg.hidden_size)[0]
            gtok, _ = gpu_dispatch_forward_token(gm, x, clock, slot, act, sli)
            r, _, _ = om.forward_token(x, clock, slot, act, sli)
            assert gtok == r, f"after kv_write: token at clock {clock}"
            assert_close(gm.read_normed_x(), om.normed_x(), what=f"after kv_write: normed x at clock {clock}")
            tok = gtok
        with pytest.raises(L.ChannelError):
            gm.kv_write(cfg.num_hidden_layers, 0, np.zeros(cfg.kv_dim, np.float32), np.zeros(cfg.kv_dim, np.float32))
    finally:
        gm.deinit()
