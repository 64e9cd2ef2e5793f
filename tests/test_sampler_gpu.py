"""The device sampler (ch_sampler_*, Sampler.sampleTopK of src/sampler.zig:217-317)
against the oracle's restatement: the reference's sampler known answers, random
candidate sets under random settings with the same generator stream (every draw
must pick the same token), and a device-resident decode loop that samples every
token on the device against a host loop of oracle forward + oracle sampler."""
import ctypes as C
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from channel_b200 import _lib as L
from tests.gpu_util import call, dev

pytestmark = pytest.mark.gpu
KATS = json.loads((Path(__file__).parent / "golden" / "reference_kats.json").read_text())


class DevSampler:
    def __init__(self, ctx, seed, temp, top_p, min_p=0.05, repeat=1.1, freq=0.1, pres=0.1, think=0, crit=0, close=0,
                 cap=4096):
        self.lib = L.load()
        p = L.ChSamplerParams(temp, top_p, min_p, repeat, freq, pres, 64, think, crit, close, 0)
        h = C.c_void_p()
        L.check(self.lib.ch_sampler_create(ctx.handle, C.byref(p), seed, cap, C.byref(h)))
        self.h, self.ctx = h.value, ctx
        self.out = torch.zeros(1, dtype=torch.int32, device="cuda")

    def sample(self, ids, vals, recent=None):
        i = dev(np.asarray(ids, np.uint32))
        v = dev(np.asarray(vals, np.float32))
        r = None if recent is None else dev(np.asarray(recent, np.uint32))
        call(self.lib.ch_sampler_sample_topk, self.h, i.data_ptr(), v.data_ptr(), len(ids),
             None if r is None else r.data_ptr(), 0 if recent is None else len(recent), self.out.data_ptr())
        self.ctx.synchronize()
        return int(self.out.item())

    def close(self):
        self.lib.ch_sampler_destroy(self.h)


@pytest.mark.parametrize("case", KATS["sampler"], ids=lambda c: c["name"][:48])
def test_sampler_kats_on_device(ctx, case):
    s = DevSampler(ctx, 42, 0.0, 0.95, repeat=case["repeat"], freq=case["freq"], pres=case["pres"],
                   think=case["think"], crit=case["crit"], close=case["close"])
    try:
        assert s.sample([c[0] for c in case["cands"]], [c[1] for c in case["cands"]], case["recent"]) == case["expect"]
    finally:
        s.close()


def test_sampler_low_temperature_kat_on_device(ctx):
    s = DevSampler(ctx, 42, 0.01, 0.95, repeat=1.2)  # src/sampler.zig:448-452
    try:
        assert s.sample([4373, 705, 1980], [18.0, 17.5, 16.0], [4373, 4373]) == 705
    finally:
        s.close()


@pytest.mark.parametrize("seed", range(6))
def test_sampler_matches_oracle_draw_for_draw(ctx, oracle, seed):
    rng = np.random.default_rng(seed)
    temp = [0.7, 1.0, 1.5, 0.3, 1.0, 2.0][seed]
    top_p = [0.95, 0.9, 1.0, 0.5, 0.99, 0.8][seed]
    min_p = [0.05, 0.0, 0.1, 0.05, 0.01, 0.2][seed]
    kw = dict(repeat=float(rng.choice([1.0, 1.1, 1.3])), freq=float(rng.choice([0.0, 0.1, 0.4])),
              pres=float(rng.choice([0.0, 0.1, 0.3])), think=int(seed == 1), crit=int(seed == 2), close=int(seed == 3))
    s = DevSampler(ctx, 1000 + seed, temp, top_p, min_p, **kw)
    o = oracle.Sampler(1000 + seed, temp, top_p, min_p, kw["repeat"], kw["freq"], kw["pres"], bool(kw["think"]),
                       bool(kw["crit"]), bool(kw["close"]))
    try:
        for it in range(40):
            n = int(rng.integers(1, 65))
            ids = rng.choice(262144, n, replace=False).astype(np.uint32)
            if it % 5 == 0:  # suppressed and critique ids among the candidates
                ids[: min(n, 3)] = rng.choice([0, 100, 101, 255999, 20470, 4573], min(n, 3), replace=False)
            vals = np.sort(rng.normal(10.0, 3.0, n).astype(np.float32))[::-1].copy()
            recent = None if it % 7 == 0 else rng.choice(np.concatenate([ids, rng.integers(0, 262144, 8)]),
                                                         int(rng.integers(1, 300))).astype(np.uint32)
            assert s.sample(ids, vals, recent) == o.sample_topk(ids, vals, recent), f"draw {it}"
    finally:
        s.close()


def test_device_loop_samples_like_host_loop(ctx, oracle):
    """ch_model_set_sampler + ch_decode_run_ring: every step's token is drawn on the
    device from that step's top-64 with the recent tokens so far (first token
    included), against forward_token + the oracle sampler on the host."""
    from channel_b200 import DynamicRingBuffer, GpuModelContext
    from tests.model_util import ring_step_lists, small_config
    from tests.test_ring_dev_gpu import DevRing
    cfg = small_config()
    gm = GpuModelContext.synthetic(ctx, cfg, 5)
    w = oracle.SyntheticWeights(cfg, 5)
    om = oracle.Model(cfg, w)
    lib = L.load()
    n, first = 20, 9
    s = DevSampler(ctx, 77, 1.0, 0.95, min_p=0.0, repeat=1.1, freq=0.1, pres=0.1)
    dr = DevRing(ctx)
    try:
        o = oracle.Sampler(77, 1.0, 0.95, 0.0, 1.1, 0.1, 0.1)
        ring_o = DynamicRingBuffer(cfg.num_hidden_layers, 0)
        tok, recent, ref = first, [first], []
        for clock in range(n):
            slot, act, sli = ring_step_lists(ring_o, cfg, clock)
            _, ids, vals = om.forward_token(oracle.embed(w.embed, [tok], cfg.hidden_size)[0], clock, slot, act, sli)
            tok = o.sample_topk(ids, vals, np.array(recent, np.uint32))
            recent.append(tok)
            ref.append(tok)
        gm.zero_state()
        ring = DynamicRingBuffer(cfg.num_hidden_layers, 0)
        dr.upload(ring)
        L.check(lib.ch_sampler_set_recent(s.h, np.array([first], np.uint32).ctypes.data_as(C.POINTER(C.c_uint32)), 1))
        L.check(lib.ch_model_set_sampler(gm.handle, s.h))
        L.check(lib.ch_decode_run_ring(gm.handle, dr.h, ring.h, first, 0, n))
        got = [int(t) for t in gm.decode_tokens(n)]
        assert got == ref, (got, ref)
        assert len(set(ref)) > 1, "the sampled stream should not be one repeated token"
        L.check(lib.ch_model_set_sampler(gm.handle, None))
        assert ctx.device_status() == 0
    finally:
        dr.close()
        s.close()
        gm.deinit()
