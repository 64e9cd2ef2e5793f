"""Small-model helpers shared by the whole-model GPU tests and smoke()."""
import numpy as np

from channel_b200.engine import ModelConfig


def small_config(**kw) -> ModelConfig:
    base = dict(vocab_size=4096, hidden_size=512, intermediate_size=1024, num_hidden_layers=3, num_attention_heads=4,
                num_key_value_heads=2, head_dim=256, rotary_dim=256, sliding_window=8,
                layer_types=[False, True, False])
    base.update(kw)
    return ModelConfig(**base)


def config3() -> ModelConfig:
    """one decoder layer, H 2048, I 8192, 8 q / 1 kv heads,
    D 256, causal full attention with theta 1e4 (vocab only feeds the LM head)."""
    return ModelConfig(vocab_size=4096, hidden_size=2048, intermediate_size=8192, num_hidden_layers=1,
                       num_attention_heads=8, num_key_value_heads=1, head_dim=256, rotary_dim=256,
                       rope_theta=1e4, rope_theta_full=1e4, sliding_window=1024, layer_types=[True])


def ring_step_lists(ring, cfg, clock):
    """What forwardToken does on the host before dispatch (src/model/forward.zig:42-45)."""
    ring.activateSlot(0, clock)
    slot = ring.getSlotIndex(clock)
    act = ring.getActiveSlotsLayer(0, clock, False, cfg.sliding_window)
    sli = ring.getActiveSlotsLayer(0, clock, True, cfg.sliding_window)
    return slot, act, sli


def topk_ids_agree(ids, rid, rvals, tol=1e-4):
    """ids must match exactly wherever the oracle's neighbouring values are separated
    by more than the numeric tolerance (closer pairs may legitimately swap).  The last
    entry's lower neighbour (the 65th value) is not in the list, so it is never clear:
    a near-tie there can swap in a candidate from below."""
    ids, rid, rvals = np.asarray(ids), np.asarray(rid), np.asarray(rvals, np.float64)
    if ids[0] != rid[0] and abs(rvals[0] - rvals[1]) > tol * max(1.0, abs(rvals[0])):
        return False
    gaps = np.abs(np.diff(rvals))
    clear = np.ones(len(ids), bool)
    clear[:-1] &= gaps > tol * np.maximum(1.0, np.abs(rvals[:-1]))
    clear[1:] &= gaps > tol * np.maximum(1.0, np.abs(rvals[1:]))
    clear[-1] = False
    return bool(np.all(ids[clear] == rid[clear])) and set(ids[:-4]) <= set(rid)


def topk_diff(ids, vals, rid, rvals):
    """(position, id, value, oracle id, oracle value) of every position where the ids differ"""
    return [(i, int(ids[i]), float(vals[i]), int(rid[i]), float(rvals[i])) for i in range(len(rid)) if ids[i] != rid[i]]
