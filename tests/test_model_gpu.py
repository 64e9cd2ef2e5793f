"""Whole-model GPU parity: the captured decode step (model_dispatch.zig order),
batched prefill (batch_dispatch.zig order) and the device-resident greedy loop
against the oracle's CPU forward on identical seeded weights.  Greedy tokens
must match bit-exactly."""
import numpy as np
import pytest

from channel_b200 import DynamicRingBuffer, GpuModelContext, gpu_dispatch_forward_token, gpu_dispatch_prefill_batch
from tests.gpu_util import assert_close
from tests.model_util import config3, ring_step_lists, small_config, topk_ids_agree

pytestmark = pytest.mark.gpu
SEED = 5


@pytest.fixture(scope="module")
def small(ctx, oracle):
    cfg = small_config()
    gm = GpuModelContext.synthetic(ctx, cfg, SEED)
    w = oracle.SyntheticWeights(cfg, SEED)
    yield cfg, gm, w
    gm.deinit()


def test_decode_steps_match_oracle(small, oracle):
    cfg, gm, w = small
    gm.zero_state()
    om = oracle.Model(cfg, w)
    ring = DynamicRingBuffer(cfg.num_hidden_layers, 0)
    tok = 17
    for clock in range(14):
        slot, act, sli = ring_step_lists(ring, cfg, clock)
        x = oracle.embed(w.embed, [tok], cfg.hidden_size)[0]
        gtok, cands = gpu_dispatch_forward_token(gm, x, clock, slot, act, sli)
        rtok, rid, rvals = om.forward_token(x, clock, slot, act, sli)
        assert gtok == rtok, f"greedy token diverged at clock {clock}"
        ids = np.array([c.id for c in cands])
        vals = np.array([c.val for c in cands])
        assert topk_ids_agree(ids, rid, rvals)
        assert np.allclose(vals, rvals, rtol=1e-3, atol=1e-3)
        assert_close(gm.read_x(), om.x(), what="residual x")
        assert_close(gm.read_normed_x(), om.normed_x(), what="normed x")
        tok = int(gtok)


def test_no_logits_path_keeps_state(small, oracle):
    cfg, gm, w = small
    gm.zero_state()
    om = oracle.Model(cfg, w)
    ring = DynamicRingBuffer(cfg.num_hidden_layers, 0)
    for clock, t in enumerate([3, 99, 2047]):
        slot, act, sli = ring_step_lists(ring, cfg, clock)
        x = oracle.embed(w.embed, [t], cfg.hidden_size)[0]
        gpu_dispatch_forward_token(gm, x, clock, slot, act, sli, topk_out=False)
        om.forward_token(x, clock, slot, act, sli)
        assert_close(gm.read_x(), om.x(), what="residual after no-logits step")


def test_prefill_then_decode_matches_oracle(small, oracle):
    cfg, gm, w = small
    gm.zero_state()
    om = oracle.Model(cfg, w)
    N = 40
    prompt = np.random.default_rng(1).integers(0, cfg.vocab_size, N).astype(np.uint32)
    ring = DynamicRingBuffer(cfg.num_hidden_layers, 0)
    prev = ring.getPrefillPrevSlots(0, 0, N)
    slots = np.concatenate([prev, [ring.getSlotIndex(c) for c in range(N)]]).astype(np.uint32)
    for c in range(N):
        for l in range(cfg.num_hidden_layers):
            ring.activateSlot(l, c)
    cands = gpu_dispatch_prefill_batch(gm, prompt, None, slots, 0, len(prev))
    X = oracle.embed(w.embed, prompt, cfg.hidden_size)
    rtok, rid, rvals = om.prefill(X, slots, 0, len(prev))
    ids = np.array([c.id for c in cands])
    assert ids[0] == rtok
    assert topk_ids_agree(ids, rid, rvals)
    assert_close(gm.read_normed_x(), om.normed_x(), what="prefill last normed x")
    tok = int(ids[0])
    for clock in range(N, N + 6):
        slot, act, sli = ring_step_lists(ring, cfg, clock)
        x = oracle.embed(w.embed, [tok], cfg.hidden_size)[0]
        gtok, _ = gpu_dispatch_forward_token(gm, x, clock, slot, act, sli)
        r, _, _ = om.forward_token(x, clock, slot, act, sli)
        assert gtok == r, f"decode after prefill diverged at clock {clock}"
        tok = int(gtok)


@pytest.mark.parametrize("N,chunk", [(1300, 1024), (700, 256)])
def test_long_prefill_in_chunks_matches_oracle(small, oracle, N, chunk):
    """Prompts past the 1,024-slot window of the sliding layers, prefilled in chunks that
    attend to the earlier ones through the ring's previous slots (the tensor-core causal
    attention: block edges, window starts and the causal diagonal inside one block).
    The tensor cores' f32 sums are not rounded like the shader's per-slot recurrence: the
    hidden state agrees to ~2e-4 relative after 700 tokens (measured on B200), inside the
    1e-3 float bar, so the top-64 ids are held exact away from near-ties at that bar."""
    cfg, gm, w = small
    gm.zero_state()
    om = oracle.Model(cfg, w)
    prompt = np.random.default_rng(N).integers(0, cfg.vocab_size, N).astype(np.uint32)
    X = oracle.embed(w.embed, prompt, cfg.hidden_size)
    ring = DynamicRingBuffer(cfg.num_hidden_layers, 0)
    for c0 in range(0, N, chunk):
        m = min(chunk, N - c0)
        prev = ring.getPrefillPrevSlots(0, c0, m)
        slots = np.concatenate([prev, ring.activateRange(c0, m)]).astype(np.uint32)
        cands = gpu_dispatch_prefill_batch(gm, prompt[c0:c0 + m], None, slots, c0, len(prev))
        rtok, rid, rvals = om.prefill(X[c0:c0 + m], slots, c0, len(prev))
        ids = np.array([c.id for c in cands])
        vals = np.array([c.val for c in cands])
        assert_close(gm.read_normed_x(), om.normed_x(), what=f"normed x after the chunk at {c0}")
        assert_close(gm.read_x(), om.x(), what=f"residual after the chunk at {c0}")
        assert ids[0] == rtok, f"greedy token of the chunk at {c0}"
        diff = [(i, int(ids[i]), float(vals[i]), int(rid[i]), float(rvals[i])) for i in range(len(ids)) if ids[i] != rid[i]]
        assert topk_ids_agree(ids, rid, rvals, tol=1e-3), f"top-64 ids of the chunk at {c0}: (pos, id, val, oracle id, val) {diff}"


def test_prefill_host_embed_equals_device_embed(small, oracle):
    cfg, gm, w = small
    prompt = [5, 6, 7, 4095, 0]
    slots = list(range(5))
    gm.zero_state()
    a = gpu_dispatch_prefill_batch(gm, prompt, w.embed.reshape(cfg.vocab_size, cfg.hidden_size), slots, 0, 0)
    gm.zero_state()
    b = gpu_dispatch_prefill_batch(gm, prompt, None, slots, 0, 0)
    assert [c.id for c in a] == [c.id for c in b]


def test_prefill_rejects_too_large(small):
    from channel_b200 import ChannelError
    cfg, gm, w = small
    with pytest.raises(ChannelError, match="CH_EBATCH"):
        gpu_dispatch_prefill_batch(gm, list(range(cfg.max_prefill_tokens + 1)), None,
                                   list(range(cfg.max_prefill_tokens + 1)), 0, 0)
    with pytest.raises(ChannelError, match="CH_EINVAL"):
        gpu_dispatch_prefill_batch(gm, [1, 2], None, [0, 4096], 0, 0)


def test_device_loop_matches_host_loop(small, oracle):
    cfg, gm, w = small
    steps, first = 12, 33
    # host loop
    gm.zero_state()
    ring = DynamicRingBuffer(cfg.num_hidden_layers, 0)
    plan, host_tokens, tok = [], [], first
    for clock in range(steps):
        slot, act, sli = ring_step_lists(ring, cfg, clock)
        plan.append((clock, slot, act, sli))
        x = oracle.embed(w.embed, [tok], cfg.hidden_size)[0]
        tok, _ = gpu_dispatch_forward_token(gm, x, clock, slot, act, sli)
        host_tokens.append(tok)
    # device loop over the same ring lists
    gm.zero_state()
    gm.decode_plan(plan)
    gm.decode_run(first, steps)
    dev_tokens = gm.decode_tokens(steps)
    assert list(dev_tokens) == host_tokens
    # and directly against the oracle's greedy stream over the same lists
    om = oracle.Model(cfg, w)
    tok, ref_tokens = first, []
    for clock, slot, act, sli in plan:
        tok, _, _ = om.forward_token(oracle.embed(w.embed, [tok], cfg.hidden_size)[0], clock, slot, act, sli)
        ref_tokens.append(tok)
    assert list(dev_tokens) == ref_tokens


def test_config3_prefill_layer(ctx, oracle):
    """one layer, 512-token causal prefill, seed 2."""
    cfg = config3()
    gm = GpuModelContext.synthetic(ctx, cfg, 2)
    try:
        w = oracle.SyntheticWeights(cfg, 2)
        om = oracle.Model(cfg, w)
        N = 512
        prompt = np.random.default_rng(2).integers(0, cfg.vocab_size, N).astype(np.uint32)
        slots = np.arange(N, dtype=np.uint32)
        cands = gpu_dispatch_prefill_batch(gm, prompt, None, slots, 0, 0)
        X = oracle.embed(w.embed, prompt, cfg.hidden_size)
        rtok, rid, rvals = om.prefill(X, slots, 0, 0)
        assert_close(gm.read_x(), om.x(), what="config3 last-token residual")
        assert_close(gm.read_normed_x(), om.normed_x(), what="config3 last-token normed x")
        k_ref = om.k_cache(0).reshape(4096, -1)[:N].view(np.float16).astype(np.float32)
        k_got = np.stack([gm.kv_read(0, s)[0] for s in range(0, N, 37)])
        assert_close(k_got, k_ref[::37], tol=2e-3, what="config3 K cache rows")
        assert cands[0].id == rtok
    finally:
        gm.deinit()
