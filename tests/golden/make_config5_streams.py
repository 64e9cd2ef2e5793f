"""Generates tests/golden/config5_streams.npz: the oracle's greedy streams for a
seeded 4-stream subset of BASELINE config 5 on the config-4 model (12B-shape Q4,
48 layers, seed 3).

Prompt lengths are uniform in [16, 64] and token ids uniform in [0, vocab)
(numpy default_rng(4): lengths first, then each prompt), short so the CPU oracle
finishes in minutes.  Every stream runs alone on the oracle with its own ring
(no anchors) and a zeroed KV cache: batched prefill of its prompt, then greedy
forward_token steps until it has N tokens (the prefill's counts as the first).
Recorded per stream:
  tokens   [4, N]       the greedy stream
  normed_x [4, 3840]    final-normed hidden state of its last step
  ids      [4, 64]      top-64 ids of its last step
  vals     [4, 64]      their softcapped values

CPU only (the checker); about 5 minutes on 8 cores and ~10 GB of RAM.
    python tests/golden/make_config5_streams.py [--tokens 8]
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

WEIGHT_SEED, PROMPT_SEED, N_STREAMS, LO, HI = 3, 4, 4, 16, 64


def prompts(vocab: int):
    rng = np.random.default_rng(PROMPT_SEED)
    lens = rng.integers(LO, HI + 1, N_STREAMS)
    return [rng.integers(0, vocab, int(n)).astype(np.uint32) for n in lens]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=8)
    ap.add_argument("--out", default=str(Path(__file__).with_name("config5_streams.npz")))
    args = ap.parse_args()
    cfg = config_12b()
    w = o.SyntheticWeights(cfg, WEIGHT_SEED)
    m = o.Model(cfg, w)
    toks, normed, last_ids, last_vals = [], [], [], []
    for s, p in enumerate(prompts(cfg.vocab_size)):
        t0 = time.time()
        m.l.or_model_reset_kv(m.h)
        ring = o.Ring(cfg.num_hidden_layers, 0)
        n = len(p)
        prev = ring.prefill_prev(0, 0, n)
        slots = np.concatenate([prev, [ring.get_slot_index(0, c) for c in range(n)]]).astype(np.uint32)
        for c in range(n):
            for layer in range(cfg.num_hidden_layers):
                ring.activate_slot(layer, c)
        tok, ids, vals = m.prefill(o.embed(w.embed, p, cfg.hidden_size), slots, 0, len(prev))
        out = [int(tok)]
        for i in range(args.tokens - 1):
            clock = n + i
            ring.activate_slot(0, clock)
            slot = ring.get_slot_index(0, clock)
            act = ring.active_list(0, clock, False, cfg.sliding_window)
            sli = ring.active_list(0, clock, True, cfg.sliding_window)
            tok, ids, vals = m.forward_token(o.embed(w.embed, [out[-1]], cfg.hidden_size)[0], clock, slot, act, sli)
            out.append(int(tok))
        toks.append(out)
        normed.append(m.normed_x())
        last_ids.append(ids.copy())
        last_vals.append(vals.copy())
        print(f"stream {s}: prompt {n}, tokens {out}, {time.time() - t0:.1f}s", flush=True)
    np.savez_compressed(args.out, tokens=np.array(toks, np.uint32), normed_x=np.stack(normed).astype(np.float32),
                        ids=np.stack(last_ids).astype(np.uint32), vals=np.stack(last_vals).astype(np.float32),
                        weight_seed=WEIGHT_SEED, prompt_seed=PROMPT_SEED, lo=LO, hi=HI)
    print("wrote", args.out)


if __name__ == "__main__":
    main()
