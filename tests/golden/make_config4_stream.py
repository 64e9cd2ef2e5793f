"""Generates tests/golden/config4_greedy.json: the oracle's greedy token stream for
BASELINE config 4 (12B-shape Q4, 48 layers, seed 3): batched prefill of a
512-token prompt of uniform ids, then greedy decode of 256 tokens with the ring
lists of DynamicRingBuffer (anchors = min(prompt, 512), sliding window 1024).

CPU only (the checker); takes ~15 minutes on 8 cores and ~10 GB of RAM.
    python tests/golden/make_config4_stream.py [--decode N]
"""
import argparse
import json
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from channel_b200.engine import config_12b  # noqa: E402  (config only; no library call)
from oracle import oracle as o  # noqa: E402

SEED, PROMPT = 3, 512


def ring_lists(ring: "o.Ring", cfg, clock):
    ring.activate_slot(0, clock)
    slot = ring.get_slot_index(0, clock)
    return slot, ring.active_list(0, clock, False, cfg.sliding_window), ring.active_list(0, clock, True,
                                                                                          cfg.sliding_window)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--decode", type=int, default=256)
    ap.add_argument("--out", default=str(Path(__file__).with_name("config4_greedy.json")))
    args = ap.parse_args()
    cfg = config_12b()
    t0 = time.time()
    w = o.SyntheticWeights(cfg, SEED)
    m = o.Model(cfg, w)
    print(f"weights {time.time() - t0:.1f}s", flush=True)
    prompt = np.random.default_rng(SEED).integers(0, cfg.vocab_size, PROMPT).astype(np.uint32)
    ring = o.Ring(cfg.num_hidden_layers, 0)
    ring.set_num_anchors(min(PROMPT, 512))
    prev = ring.prefill_prev(0, 0, PROMPT)
    slots = np.concatenate([prev, [ring.get_slot_index(0, c) for c in range(PROMPT)]]).astype(np.uint32)
    for c in range(PROMPT):
        for l in range(cfg.num_hidden_layers):
            ring.activate_slot(l, c)
    t0 = time.time()
    tok, ids, vals = m.prefill(o.embed(w.embed, prompt, cfg.hidden_size), slots, 0, len(prev))
    print(f"prefill {time.time() - t0:.1f}s first token {tok}", flush=True)
    stream, margins, top_ids = [int(tok)], [float(vals[0] - vals[1])], [ids[:8].tolist()]
    t0 = time.time()
    for i in range(args.decode):
        clock = PROMPT + i
        slot, act, sli = ring_lists(ring, cfg, clock)
        x = o.embed(w.embed, [stream[-1]], cfg.hidden_size)[0]
        tok, ids, vals = m.forward_token(x, clock, slot, act, sli)
        stream.append(int(tok))
        margins.append(float(vals[0] - vals[1]))
        top_ids.append(ids[:8].tolist())
        if i % 16 == 0:
            print(f"decode {i} tok {tok} margin {margins[-1]:.4g} {time.time() - t0:.1f}s", flush=True)
    out = {"config": "config4 12B-shape Q4, 48 layers, seed 3, prompt 512 uniform ids (numpy default_rng(3)), "
                     "anchors 512, sliding window 1024",
           "prompt_seed": SEED, "prompt_len": PROMPT,
           "tokens": stream, "top1_top2_margin": margins, "top8_ids": top_ids,
           "note": "tokens[0] comes from prefill; tokens[i] (i>=1) is the greedy token decoded at clock 511+i"}
    Path(args.out).write_text(json.dumps(out) + "\n")
    print("wrote", args.out)


if __name__ == "__main__":
    main()
