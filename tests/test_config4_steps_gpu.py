"""Config 4 step by step: the 12B-shape Q4 model (48 layers, synthetic seed-3 weights)
through the reference-facing calls -- ch_prefill for the 512-token prompt, then
ch_forward_token per token with the embedding row built on the host like
forward.zig:33-37 -- against the oracle's values committed in
tests/golden/config4_steps.npz (tests/golden/make_config4_steps.py).

The greedy stream alone says little at this shape (random-init weights repeat one
token), so every step also checks what produced it: the top-64 ids (exact wherever
the oracle's neighbouring values are more than 1e-3 apart), their softcapped values
and the final-normed hidden state the LM head read (1e-3 relative), and the residual
after the prefill and after the last step."""
from pathlib import Path

import numpy as np
import pytest

from channel_b200 import DynamicRingBuffer, GpuModelContext, gpu_dispatch_forward_token, gpu_dispatch_prefill_batch
from channel_b200 import _lib as L
from channel_b200.engine import config_12b
from tests.gpu_util import assert_close
from tests.model_util import ring_step_lists, topk_ids_agree

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).with_name("golden") / "config4_steps.npz"
TOL = 1e-3


def _host_embedding(ctx, cfg, seed):
    """the model's bf16 table, generated on the device (same generator as the model) and
    copied to the host: what the reference's host keeps mmap'd (safetensors.zig:139)"""
    import torch
    lib = L.load()
    t = torch.empty(cfg.vocab_size * cfg.hidden_size, dtype=torch.int16, device="cuda")
    L.check(lib.ch_gen_bf16(ctx.handle, t.data_ptr(), t.numel(), lib.ch_tensor_seed(seed, 0, 20), 0.0, 0.02))
    ctx.synchronize()
    return t.cpu().numpy().view(np.uint16).reshape(cfg.vocab_size, cfg.hidden_size)


def test_config4_prefill_and_steps_match_oracle_values(ctx):
    g = np.load(GOLDEN)
    seed, n_prompt = int(g["prompt_seed"]), int(g["prompt_len"])
    cfg = config_12b()
    gm = GpuModelContext.synthetic(ctx, cfg, seed)
    ring = DynamicRingBuffer(cfg.num_hidden_layers, 0)
    try:
        table = _host_embedding(ctx, cfg, seed)
        scale = np.float32(np.sqrt(cfg.hidden_size))
        prompt = np.random.default_rng(seed).integers(0, cfg.vocab_size, n_prompt).astype(np.uint32)
        ring.setNumAnchors(min(n_prompt, 512))
        prev = ring.getPrefillPrevSlots(0, 0, n_prompt)
        slots = np.concatenate([prev, [ring.getSlotIndex(c) for c in range(n_prompt)]]).astype(np.uint32)
        for c in range(n_prompt):
            for layer in range(cfg.num_hidden_layers):
                ring.activateSlot(layer, c)
        cands = gpu_dispatch_prefill_batch(gm, prompt, None, slots, 0, len(prev))

        def check(step, cands, what):
            ids = np.array([c.id for c in cands])
            vals = np.array([c.val for c in cands], np.float32)
            assert ids[0] == g["tokens"][step], f"{what}: greedy token"
            assert topk_ids_agree(ids, g["ids"][step], g["vals"][step], tol=TOL), f"{what}: top-64 ids"
            np.testing.assert_allclose(vals, g["vals"][step], rtol=TOL, atol=TOL, err_msg=f"{what}: top-64 values")
            assert_close(gm.read_normed_x(), g["normed_x"][step], tol=TOL, what=f"{what}: normed x")

        check(0, cands, "prefill")
        assert_close(gm.read_x(), g["x"][0], tol=TOL, what="prefill: residual")
        n_steps = len(g["tokens"]) - 1
        for i in range(n_steps):
            clock = n_prompt + i
            slot, act, sli = ring_step_lists(ring, cfg, clock)
            x = (table[int(g["tokens"][i])].astype(np.uint32) << 16).view(np.float32) * scale
            _, cands = gpu_dispatch_forward_token(gm, x, clock, slot, act, sli)
            check(i + 1, cands, f"decode step {i} (clock {clock})")
        assert_close(gm.read_x(), g["x"][1], tol=TOL, what="residual after the last step")
        assert ctx.device_status() == 0
    finally:
        gm.deinit()
        ring.deinit()
