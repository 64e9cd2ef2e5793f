"""Per-phase timeline of the decode-step kernel (a profiling aid).

Loads the instrumented library (``python -m channel_b200.build --trace`` builds
libchannel_b200_trace.so with -DCH_PHASE_TRACE), decodes a few greedy tokens of
the 12B-shape model on synthetic weights and prints, per phase kind, where the
time of one token goes.  Each CTA's thread 0 records %globaltimer at these
points of every phase (marks 8-11, from warps 0 and 15 inside the tile loop, are
saved by --dump, as is mark 12 of phase 0, the CTA's SM id):

  0 phase start (grid barrier passed)    1 staged inputs landed (bulk copies)
  2 GEMV: input limbs built / ATTN: heads normed and roped
  3 GEMV: weight tiles done / ATTN: split partial written
  4 phase done (GEMV: CTA combine; ATTN: split combine)
  5 arrived at the next barrier and issued the next phase's early copies
  6 next barrier passed
  7 (inside the prologue) GEMV add+norm: straddling rows patched / ATTN: q|k|v rows patched

A phase's cost is taken from the slowest CTA at each point (the grid waits for
it); the per-CTA table shows median / max of each interval for layer 1.
Usage (one GPU):

  python bench_phases.py [--layers 48] [--steps 4] [--clock 599] [--lib PATH]
  torchrun --nproc-per-node N bench_phases.py   # tensor parallel, rank 0 prints
"""
from __future__ import annotations

import argparse
import collections
import ctypes as C
from pathlib import Path

import numpy as np

TRACE_CTAS, TRACE_PHASES, TRACE_MARKS = 256, 512, 13
COLS = ["staging", "prologue", "tiles/core", "combine", "arrive+pre", "barrier"]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--clock", type=int, default=599, help="decode position (active slots = clock + 1)")
    ap.add_argument("--lib", default=None, help="an already built instrumented library (default: build it)")
    ap.add_argument("--dump", default=None, help="also save the raw [cta][phase][8 marks] ns array (.npy)")
    args = ap.parse_args()

    from channel_b200 import _lib as L
    from channel_b200 import build

    L.LIB_PATH = Path(args.lib) if args.lib else build.build(trace=True)
    lib = L.load()
    lib.ch_phase_trace_copy.restype = C.c_int
    lib.ch_phase_trace_copy.argtypes = [C.c_void_p, C.c_size_t]

    import torch

    from channel_b200 import DynamicRingBuffer, GpuContext, GpuModelContext, config_12b
    from channel_b200.engine import gpu_dispatch_forward_token

    import os
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    torch.cuda.set_device(rank)
    ctx = GpuContext.init(rank)
    cfg = config_12b(layers=args.layers)
    if world > 1:  # tensor parallel under torchrun: every rank traces, rank 0 prints
        import torch.distributed as dist

        from channel_b200.engine import attach_tensor_parallel
        dist.init_process_group("gloo")
        gm = GpuModelContext.synthetic_sharded(ctx, cfg, 3, rank, world)
        attach_tensor_parallel(gm)
        dist.barrier()
    else:
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
    grid = min(TRACE_CTAS, torch.cuda.get_device_properties(rank).multi_processor_count)
    nph = 5 * cfg.num_hidden_layers + (3 if world > 1 else 2)
    if rank != 0:
        if world > 1:
            dist.barrier()
        gm.deinit()
        ctx.deinit()
        return
    if args.dump:
        np.save(args.dump, buf.reshape(TRACE_CTAS, TRACE_PHASES, TRACE_MARKS)[:grid, :nph])
    tr = buf.reshape(TRACE_CTAS, TRACE_PHASES, TRACE_MARKS)[:grid, :nph, :7].astype(np.int64)
    kinds = ["qkv", "attn", "o", "gateup", "down"]

    def fill(t, pi):
        """marks a phase kind (or CTA) does not record take the previous mark's time"""
        t = t.copy()
        last = pi == nph - 1
        for k in range(1, 7):
            if last and k >= 5:
                t[..., k] = t[..., 4]
            else:
                t[..., k] = np.where(t[..., k] == 0, t[..., k - 1], t[..., k])
        return t

    agg = collections.defaultdict(lambda: np.zeros(6))
    cnt = collections.Counter()
    for pi in range(nph):
        tail = ["lm", "topk", "merge"]
        kind = kinds[pi % 5] if pi < 5 * cfg.num_hidden_layers else tail[pi - 5 * cfg.num_hidden_layers]
        st = fill(tr[:, pi, :], pi)
        agg[kind] += np.diff(st.max(axis=0))  # slowest CTA at each mark
        cnt[kind] += 1
    span = tr[:, nph - 1, 4].max() - tr[:, 0, 0].min()
    print(f"decode step span {span / 1e3:.1f} us ({cfg.num_hidden_layers} layers, clock {args.clock}, "
          f"{len(act)} active / {len(sli)} sliding slots)")
    print("phase   n   " + "".join(f"{c:>12s}" for c in COLS) + "   (us per phase, slowest CTA)")
    for k in ["qkv", "attn", "o", "gateup", "down", "lm", "topk"] + (["merge"] if world > 1 else []):
        a = agg[k] / max(cnt[k], 1) / 1e3
        print(f"{k:7s} {cnt[k]:3d} " + "".join(f"{v:12.2f}" for v in a))
    per_layer = sum(agg[k].sum() for k in kinds) / cfg.num_hidden_layers / 1e3
    print(f"per layer {per_layer:.2f} us")
    print("layer 1, per CTA (median / max us):")
    for j, k in enumerate(kinds):
        pi = 5 + j
        d = np.diff(fill(tr[:, pi, :], pi), axis=1) / 1e3
        med, mx = np.median(d, axis=0), d.max(axis=0)
        print(f"  {k:7s} " + "  ".join(f"{a:5.2f}/{b:5.2f}" for a, b in zip(med, mx)))
    if world > 1:
        dist.barrier()
    gm.deinit()
    ctx.deinit()


if __name__ == "__main__":
    main()
