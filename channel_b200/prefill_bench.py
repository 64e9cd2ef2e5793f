"""Batched prefill timing on the 12B-shape synthetic model (a measurement and
profiling aid): a prompt of uniform-random token ids goes through
gpu_dispatch_prefill_batch, timed with CUDA events on the library's stream.

  python -m channel_b200.prefill_bench [--tokens 512] [--reps 3] [--layers 48]
"""
from __future__ import annotations

import argparse

import numpy as np


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=512)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--layers", type=int, default=48)
    args = ap.parse_args()

    import torch

    from channel_b200 import DynamicRingBuffer, GpuContext, GpuModelContext, config_12b, gpu_dispatch_prefill_batch
    cfg = config_12b(layers=args.layers)
    ctx = GpuContext.init(0)
    gm = GpuModelContext.synthetic(ctx, cfg, 3)
    stream = torch.cuda.ExternalStream(ctx.stream)
    n = args.tokens
    prompt = np.random.default_rng(3).integers(0, cfg.vocab_size, n).astype(np.uint32)
    times = []
    for _ in range(args.reps + 1):
        gm.zero_state()
        ring = DynamicRingBuffer(cfg.num_hidden_layers, 0)
        prev = ring.getPrefillPrevSlots(0, 0, n)
        slots = np.concatenate([prev, [ring.getSlotIndex(c) for c in range(n)]]).astype(np.uint32)
        ctx.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        cands = gpu_dispatch_prefill_batch(gm, prompt, None, slots, 0, len(prev))
        e1.record(stream)
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    best = min(times[1:])
    print(f"prefill {n} tokens, {cfg.num_hidden_layers} layers: {best:.2f} ms ({n / best * 1e3:.0f} tok/s), "
          f"first token {int(cands[0].id)}, device status {ctx.device_status()}", flush=True)
    gm.deinit()
    ctx.deinit()


if __name__ == "__main__":
    main()
