"""Per-phase timeline of the decode-step kernel (a profiling aid).

Loads the instrumented library (``python -m channel_b200.build --trace`` builds
libchannel_b200_trace.so with -DCH_PHASE_TRACE), decodes a few greedy tokens of
the 12B-shape model on synthetic weights and prints, per phase kind, where the
time of one token goes.  Each CTA's thread 0 records %globaltimer at six points
of every phase:

  0 phase start (after the barrier)   1 input prologue done   2 weight tiles done
  3 phase done                        4 next phase's pre-loads issued   5 barrier passed

A phase's cost is taken from the slowest CTA at each point (the grid waits for
it).  Usage (one GPU):

  python -m channel_b200.phase_trace [--layers 48] [--steps 4] [--clock 599] [--lib PATH]
"""
from __future__ import annotations

import argparse
import collections
import ctypes as C

import numpy as np

TRACE_CTAS, TRACE_PHASES, TRACE_MARKS = 256, 512, 6


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--clock", type=int, default=599, help="decode position (active slots = clock + 1)")
    ap.add_argument("--lib", default=None, help="an already built instrumented library (default: build it)")
    args = ap.parse_args()

    from pathlib import Path

    from channel_b200 import _lib as L
    from channel_b200 import build

    L.LIB_PATH = Path(args.lib) if args.lib else build.build(trace=True)
    lib = L.load()
    lib.ch_phase_trace_copy.restype = C.c_int
    lib.ch_phase_trace_copy.argtypes = [C.c_void_p, C.c_size_t]

    from channel_b200 import DynamicRingBuffer, GpuContext, GpuModelContext, config_12b
    from channel_b200.engine import gpu_dispatch_forward_token

    ctx = GpuContext.init(0)
    cfg = config_12b(layers=args.layers)
    gm = GpuModelContext.synthetic(ctx, cfg, 3)
    ring = DynamicRingBuffer(cfg.num_hidden_layers, 0)
    x = np.random.default_rng(0).standard_normal(cfg.hidden_size).astype(np.float32)
    for c in range(args.clock + 1):
        ring.activateSlot(0, c)
    act = ring.getActiveSlotsLayer(0, args.clock, False, cfg.sliding_window)
    sli = ring.getActiveSlotsLayer(0, args.clock, True, cfg.sliding_window)
    for _ in range(args.steps):
        gpu_dispatch_forward_token(gm, x, args.clock, args.clock % 4096, act, sli)
    ctx.synchronize()
    buf = np.zeros(TRACE_CTAS * TRACE_PHASES * TRACE_MARKS, np.uint64)
    L.check(lib.ch_phase_trace_copy(buf.ctypes.data, buf.size))
    grid = min(TRACE_CTAS, gm_grid())
    nph = 5 * cfg.num_hidden_layers + 2
    tr = buf.reshape(TRACE_CTAS, TRACE_PHASES, TRACE_MARKS)[:grid, :nph, :].astype(np.int64)
    kinds = ["qkv", "attn", "o", "gateup", "down"]
    cols = ["prologue", "tiles", "combine/attn", "pre-loads", "barrier"]
    agg = collections.defaultdict(lambda: np.zeros(5))
    cnt = collections.Counter()
    for pi in range(nph):
        kind = kinds[pi % 5] if pi < 5 * cfg.num_hidden_layers else ("lm" if pi == nph - 2 else "topk")
        st = tr[:, pi, :].max(axis=0)  # slowest CTA at each mark
        if kind in ("attn", "topk"):
            st[1] = st[2] = st[0]
        if pi == nph - 1:
            st[4] = st[5] = st[3]
        agg[kind] += np.diff(st)
        cnt[kind] += 1
    span = tr[:, nph - 1, 3].max() - tr[:, 0, 0].min()
    print(f"decode step span {span / 1e3:.1f} us ({cfg.num_hidden_layers} layers, clock {args.clock}, "
          f"{len(act)} active / {len(sli)} sliding slots)")
    print("phase   n    " + "  ".join(f"{c:>12s}" for c in cols) + "   (us per phase, slowest CTA)")
    for k in ["qkv", "attn", "o", "gateup", "down", "lm", "topk"]:
        a = agg[k] / max(cnt[k], 1) / 1e3
        print(f"{k:7s} {cnt[k]:3d}  " + "  ".join(f"{v:12.2f}" for v in a))
    per_layer = sum(agg[k].sum() for k in kinds) / cfg.num_hidden_layers / 1e3
    print(f"per layer {per_layer:.2f} us")
    # per-CTA spread of layer 1's phases: median / max over CTAs of each interval
    print("layer 1, per CTA (median / max us):")
    for j, k in enumerate(kinds):
        pi = 5 + j
        d = np.diff(tr[:, pi, :], axis=1) / 1e3
        if k == "attn":
            d[:, 0] = d[:, 1] = 0.0
            d[:, 2] = (tr[:, pi, 3] - tr[:, pi, 0]) / 1e3
        med, mx = np.median(d, axis=0), d.max(axis=0)
        print(f"  {k:7s} " + "  ".join(f"{a:6.2f}/{b:6.2f}" for a, b in zip(med, mx)) +
              f"   slowest prologue CTA {int(d[:, 0].argmax())}, slowest tiles CTA {int(d[:, 1].argmax())}")
    gm.deinit()
    ctx.deinit()


def gm_grid() -> int:
    import torch
    return torch.cuda.get_device_properties(0).multi_processor_count


if __name__ == "__main__":
    main()
