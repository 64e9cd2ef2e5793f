"""Generates tests/golden/config4_steps.npz: per-step values of the oracle's config-4
run (12B-shape Q4, 48 layers, seed 3) that pin more than the greedy token stream.

Same workload as make_config4_stream.py -- batched prefill of a 512-token prompt of
uniform ids, then greedy decode with the ring lists of DynamicRingBuffer (anchors =
min(prompt, 512), sliding window 1024) -- but for the prefill and the first N decode
steps it records:
  tokens   [N+1]        greedy token (row 0: the prefill's)
  ids      [N+1, 64]    top-64 ids (softcapped logits, value desc, lowest id first)
  vals     [N+1, 64]    their softcapped values
  normed_x [N+1, 3840]  final-normed hidden state the LM head reads
  x        [2, 3840]    residual after the prefill and after the last step

CPU only (the checker); about 3 minutes on 8 cores and ~10 GB of RAM.
    python tests/golden/make_config4_steps.py [--decode 16]
"""
import argparse
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from channel_b200.engine import config_12b  # noqa: E402  (config only; no library call)
from oracle import oracle as o  # noqa: E402

SEED, PROMPT = 3, 512


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--decode", type=int, default=16)
    ap.add_argument("--out", default=str(Path(__file__).with_name("config4_steps.npz")))
    args = ap.parse_args()
    cfg = config_12b()
    w = o.SyntheticWeights(cfg, SEED)
    m = o.Model(cfg, w)
    prompt = np.random.default_rng(SEED).integers(0, cfg.vocab_size, PROMPT).astype(np.uint32)
    ring = o.Ring(cfg.num_hidden_layers, 0)
    ring.set_num_anchors(min(PROMPT, 512))
    prev = ring.prefill_prev(0, 0, PROMPT)
    slots = np.concatenate([prev, [ring.get_slot_index(0, c) for c in range(PROMPT)]]).astype(np.uint32)
    for c in range(PROMPT):
        for layer in range(cfg.num_hidden_layers):
            ring.activate_slot(layer, c)
    t0 = time.time()
    tok, ids, vals = m.prefill(o.embed(w.embed, prompt, cfg.hidden_size), slots, 0, len(prev))
    print(f"prefill {time.time() - t0:.1f}s first token {tok}", flush=True)
    tokens, all_ids, all_vals, normed, xs = [int(tok)], [ids.copy()], [vals.copy()], [m.normed_x()], [m.x()]
    for i in range(args.decode):
        clock = PROMPT + i
        ring.activate_slot(0, clock)
        slot = ring.get_slot_index(0, clock)
        act = ring.active_list(0, clock, False, cfg.sliding_window)
        sli = ring.active_list(0, clock, True, cfg.sliding_window)
        x = o.embed(w.embed, [tokens[-1]], cfg.hidden_size)[0]
        tok, ids, vals = m.forward_token(x, clock, slot, act, sli)
        tokens.append(int(tok))
        all_ids.append(ids.copy())
        all_vals.append(vals.copy())
        normed.append(m.normed_x())
        print(f"decode {i} tok {tok} margin {vals[0] - vals[1]:.4g}", flush=True)
    xs.append(m.x())
    np.savez_compressed(args.out, tokens=np.array(tokens, np.uint32), ids=np.stack(all_ids).astype(np.uint32),
                        vals=np.stack(all_vals).astype(np.float32), normed_x=np.stack(normed).astype(np.float32),
                        x=np.stack(xs).astype(np.float32), prompt_seed=SEED, prompt_len=PROMPT)
    print("wrote", args.out)


if __name__ == "__main__":
    main()
