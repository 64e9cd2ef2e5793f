"""Multi-stream greedy decode (BASELINE config 5's path) against the oracle.

Streams with ragged prompts share one model; each has its own ring and KV cache.
Steps pack up to max_batch streams per launch (four streams at three per launch
take two launches a round; 9 and 17 streams in one launch run the batched LM head
with padded token groups) and every stream must reproduce, token for token, the
greedy stream the oracle produces for it alone (prefill, then forward_token)."""
import numpy as np
import pytest

from channel_b200 import _lib as L
from tests.model_util import ring_step_lists, small_config

pytestmark = pytest.mark.gpu

SEED = 7
N_TOKENS = 6


def _oracle_stream(oracle, cfg, w, prompt, n_tokens):
    from channel_b200 import DynamicRingBuffer
    om = oracle.Model(cfg, w)
    ring = DynamicRingBuffer(cfg.num_hidden_layers, 0)
    n = len(prompt)
    prev = ring.getPrefillPrevSlots(0, 0, n)
    slots = np.concatenate([prev, [ring.getSlotIndex(c) for c in range(n)]]).astype(np.uint32)
    for c in range(n):
        for layer in range(cfg.num_hidden_layers):
            ring.activateSlot(layer, c)
    t, _, _ = om.prefill(oracle.embed(w.embed, prompt, cfg.hidden_size), slots, 0, len(prev))
    out = [int(t)]
    for i in range(n_tokens - 1):
        clock = n + i
        slot, act, sli = ring_step_lists(ring, cfg, clock)
        t, _, _ = om.forward_token(oracle.embed(w.embed, [int(t)], cfg.hidden_size)[0], clock, slot, act, sli)
        out.append(int(t))
    return out


@pytest.mark.parametrize("n_streams,max_batch", [(4, 3), (9, 9), (17, 17)])
def test_streams_match_oracle(ctx, oracle, n_streams, max_batch):
    from channel_b200 import GpuModelContext
    from channel_b200.streams import MultiStreamDecoder
    cfg = small_config()
    rng = np.random.default_rng(11 + n_streams)
    lens = rng.integers(1, 20, n_streams)
    prompts = [rng.integers(0, cfg.vocab_size, n).astype(np.uint32) for n in lens]
    w = oracle.SyntheticWeights(cfg, SEED)
    refs = [_oracle_stream(oracle, cfg, w, p, N_TOKENS) for p in prompts]
    gm = GpuModelContext.synthetic(ctx, cfg, SEED)
    dec = MultiStreamDecoder(gm, cfg, n_streams=n_streams, max_batch=max_batch)
    got = dec.run(prompts, N_TOKENS)
    for s, (g, r) in enumerate(zip(got, refs)):
        assert g == r, f"stream {s}: {g} != oracle {r}"
    assert dec.steps == -(-n_streams // max_batch) * (N_TOKENS - 1)
    assert ctx.device_status() == 0
    gm.deinit()


def test_streams_reject_bad_steps(ctx):
    from channel_b200 import GpuModelContext
    cfg = small_config()
    gm = GpuModelContext.synthetic(ctx, cfg, SEED)
    gm.streams_init(2, 2)
    lib = L.load()
    with pytest.raises(L.ChannelError):
        gm.streams_init(2, 2)  # twice
    dup = [(0, 1, 0, 0, [0], [0]), (0, 2, 0, 0, [0], [0])]
    with pytest.raises(L.ChannelError) as e:
        gm.streams_decode(dup)
    assert e.value.status == L.CH_EINVAL
    three = [(i % 2, 1, 0, 0, [0], [0]) for i in range(3)]
    with pytest.raises(L.ChannelError) as e:
        gm.streams_decode(three)
    assert e.value.status == L.CH_EBATCH
    with pytest.raises(L.ChannelError) as e:
        gm.streams_decode([(2, 1, 0, 0, [0], [0])])
    assert e.value.status == L.CH_EINVAL
    assert b"stream" in lib.ch_last_error()
    gm.deinit()


def test_config5_12b_streams_match_oracle_golden(ctx):
    """A seeded 4-stream subset of BASELINE config 5 on the 12B-shape model (48 layers,
    seed-3 weights): prompts of 16-64 ids, 8 greedy tokens each, all four streams in
    every batched step.  Against tests/golden/config5_streams.npz (the oracle running
    each stream alone, tests/golden/make_config5_streams.py): every token, the last
    step's final-normed hidden state per stream (1e-3 relative) and the top-8 of its
    softcapped logits (ids exact away from near-ties, values within 1e-3)."""
    from pathlib import Path

    from channel_b200 import GpuModelContext
    from channel_b200.engine import config_12b
    from channel_b200.streams import MultiStreamDecoder
    from tests.gpu_util import assert_close
    from tests.model_util import topk_ids_agree

    g = np.load(Path(__file__).with_name("golden") / "config5_streams.npz")
    cfg = config_12b()
    rng = np.random.default_rng(int(g["prompt_seed"]))
    n_streams, n_tokens = g["tokens"].shape
    lens = rng.integers(int(g["lo"]), int(g["hi"]) + 1, n_streams)
    prompts = [rng.integers(0, cfg.vocab_size, int(n)).astype(np.uint32) for n in lens]
    gm = GpuModelContext.synthetic(ctx, cfg, int(g["weight_seed"]))
    try:
        dec = MultiStreamDecoder(gm, cfg, n_streams=n_streams, max_batch=n_streams)
        got = dec.run(prompts, n_tokens)
        for s in range(n_streams):
            assert got[s] == [int(t) for t in g["tokens"][s]], f"stream {s}: {got[s]} != {g['tokens'][s].tolist()}"
        normed = gm.streams_read_normed_x(n_streams)
        logits = gm.streams_read_logits(n_streams).astype(np.float64)
        for s in range(n_streams):
            assert_close(normed[s], g["normed_x"][s], what=f"stream {s}: last step's normed x")
            capped = 30.0 * np.tanh(logits[s] / 30.0)
            top = np.lexsort((np.arange(cfg.vocab_size), -capped))[:8]
            assert topk_ids_agree(top, g["ids"][s][:8], g["vals"][s][:8], tol=1e-3), f"stream {s}: top-8 ids"
            np.testing.assert_allclose(capped[top], g["vals"][s][:8], rtol=1e-3, atol=1e-3)
        assert ctx.device_status() == 0
    finally:
        gm.deinit()
