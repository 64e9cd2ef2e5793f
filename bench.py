#!/usr/bin/env python
"""bench.py -- decode tok/s of the 12B-shape Q4 model on B200.

One "step" = one greedy decode token through all 48 layers + the Q8 LM head +
top-64 (the reference's gpuDispatchForwardToken, src/gpu/model_dispatch.zig:128-153).
Workload: seeded synthetic weights (seed 3), a 512-token prompt of uniform ids
prefilled with the batched path, then greedy decode at clocks 512.. (config 4
decodes 256 tokens; warmup + steps default to 8 + 248 = 256).  Per-token weight
stream is 7.2 GB (> 126 MB L2), so no L2 flush is needed between steps.

  value : device-resident loop (ch_decode_run_ring: each step's ring lists built on the
          device, the greedy token fed back on the device), CUDA events on the library
          stream.
  e2e   : the reference-facing call ch_forward_token per token with host buffers
          (x from the host bf16 table, host ring lists, top-64 read back).
  --impl reference : the reference CPU path = the oracle restatement (Zig cannot
          be built here), all host threads, one bounded sample per step.

Multi-GPU (torchrun): row-sharded tensor parallel -- all ranks decode the same
token stream, each with 1/N of the weights (q|k|v and KV by heads, o / down by
output rows, gate|up by intermediate rows, LM head by vocab rows); the persistent
decode kernel writes each phase's outputs straight into every rank's memory over
NVLink and the ranks meet at one arrival counter per phase (strong scaling).
The prefill runs token by token through the same kernel.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

SEED = 3
PROMPT = 512


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=248)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-config5", action="store_true", help="skip the multi-stream (config 5) measurement")
    ap.add_argument("--config5-streams", type=int, default=64)
    ap.add_argument("--kernel-only", action="store_true",
                    help="only time the dominant kernel (fused gate/up GEMV) over rotating layers; for ncu captures")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks + throttle reasons sampled during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.proc = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append([s.strip() for s in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if len(s) > 8 and s[1].replace(".", "").isdigit()]
        smax = [float(s[2]) for s in self.samples if len(s) > 8 and s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples if len(s) > 8 for i in range(4) if s[5 + i] == "Active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(self.samples)}


# ----------------------------------------------------------------------------------------
def cpu_model_name() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_sample(steps: int, warmup: int):
    """Reference CPU path (the oracle restatement, all host threads) on the full config-4
    decode step: all 48 layers (every 5th one full attention over the whole list, the
    others over the 1,024-slot sliding window), the whole Q8 LM head and the top-64, one
    greedy token per step at clocks 512, 513, ... with the token fed back.  The prompt's
    K/V rows are not prefilled on the CPU (minutes of work): they stay zero, which reads
    and multiplies exactly the same rows as a prefilled cache."""
    from channel_b200.engine import config_12b
    from oracle import oracle as o

    cfg = config_12b()
    t0 = time.perf_counter()
    w = o.SyntheticWeights(cfg, SEED)
    m = o.Model(cfg, w)
    setup_s = time.perf_counter() - t0
    ring = o.Ring(cfg.num_hidden_layers, 0)
    ring.set_num_anchors(PROMPT)
    for c in range(PROMPT):
        ring.activate_slot(0, c)
    tok = int(np.random.default_rng(SEED).integers(0, cfg.vocab_size))
    times = []
    for i in range(warmup + steps):
        clock = PROMPT + i
        ring.activate_slot(0, clock)
        slot = ring.get_slot_index(0, clock)
        act = ring.active_list(0, clock, False, cfg.sliding_window)
        sli = ring.active_list(0, clock, True, cfg.sliding_window)
        x = o.embed(w.embed, [tok], cfg.hidden_size)[0]
        t0 = time.perf_counter()
        tok, _, _ = m.forward_token(x, clock, slot, act, sli)
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
    t_tok = float(np.mean(times))
    del m, w
    return {"value": 1.0 / t_tok, "unit": "tok/s", "cores": o.nthreads(), "cpu_model": cpu_model_name(),
            "kind": "port",
            "sample": "oracle greedy decode of the whole config-4 step (48 layers, Q8 LM head over 262,144 rows, "
                      "top-64) at clocks {}..{}: mean of {} tokens after {} warm-up".format(
                          PROMPT + warmup, PROMPT + warmup + steps - 1, steps, warmup),
            "sec_per_token": t_tok, "setup_s": setup_s, "timed_s": float(np.sum(times))}


def workload_config(layers: int, n_total: int) -> dict:
    """The config both arms report: the config-4 decode workload, K + W tokens after the prompt."""
    return {"workload": "config4: 12B-shape Q4 greedy decode ({} layers, H 3840, I 15360, 16q/8kv heads, "
                        "D 256, V 262144 Q8 head) after a 512-token prefill, seed 3".format(layers),
            "global_batch": 1, "seq_len": PROMPT + n_total}


def reference_arm(args):
    """The reference's CPU path (the oracle port, all host threads) on the same workload:
    W warm-up tokens, then K timed tokens, each a whole config-4 decode step (~1 s on
    16 cores, so the driver's K = 20, W = 5 run takes well under a minute)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    steps = max(1, args.steps)
    warm = max(0, args.warmup)
    r = cpu_sample(steps, warm)
    line = {"metric": "decode tok/s (12B-shape Q4) at 1/2/4/8 GPU; Q4 GEMV HBM GB/s vs peak",
            "impl": "reference", "value": r["value"], "unit": "tok/s", "n_gpus": args.gpus, "steps": steps,
            "warmup": warm, "ms_per_step": 1000.0 / r["value"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {**workload_config(48, warm + steps), "parallelism": "cpu (the oracle port on the host cores)"},
            "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "cpu_model", "kind", "sample")},
            "e2e": {"value": r["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------------------
def time_launches(ctx, stream, call, n):
    """Device time per launch of n back-to-back calls (call(i) enqueues launch i on the
    library stream).  The stream first waits behind a short device sleep on torch's
    stream, so every launch is queued before the first runs: the events then time the
    kernels, not the host's call rate."""
    import torch
    ctx.synchronize()
    torch.cuda.synchronize()
    torch.cuda._sleep(int(4e6))  # a few ms of device time (clock cycles)
    stream.wait_stream(torch.cuda.current_stream())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(n):
        call(i)
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / n


def gateup_roofline(ctx, gm, cfg, stream, reps=3):
    """Dominant decode kernel (fused gate/up Q4 GEMV + GELU*up, 53% of the weight bytes)
    timed alone through ch_fused_mlp_q4 with CUDA events on the library stream, rotating
    over every layer's weights so no launch finds its 66 MB in L2."""
    import torch
    from channel_b200 import _lib as L
    lib = L.load()
    H, I = cfg.hidden_size, cfg.intermediate_size
    xbuf = torch.randn(H, device="cuda", dtype=torch.float32)
    ybuf = torch.empty(I, device="cuda", dtype=torch.float32)
    tiles = [gm.weight_tiles(l, 2)[0] for l in range(cfg.num_hidden_layers)]
    torch.cuda.synchronize()

    def call(i):
        L.check(lib.ch_fused_mlp_q4(ctx.handle, tiles[i % len(tiles)], I, H, xbuf.data_ptr(), ybuf.data_ptr()))
    for i in range(len(tiles)):
        call(i)
    n = reps * len(tiles)
    k_ms = time_launches(ctx, stream, call, n)
    nbytes = 2 * I * H * 18 // 32 + H * 4 + I * 4
    peak, peak_kind = peaks()
    achieved = nbytes / (k_ms / 1000.0) / 1e9
    traffic = None
    tp = ROOT / "profiles" / "gemv_gateup_traffic.json"
    if tp.exists():
        traffic = json.loads(tp.read_text()).get("bytes_per_launch")
    return {"bound": "hbm", "kernel": "gemv_kernel<Q4, GELU_MUL> (fused gate/up, 2x15360x3840)",
            "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak, "traffic": traffic,
            "bytes_per_launch": nbytes, "us_per_launch": k_ms * 1000, "launches_timed": n,
            "peak_kind": peak_kind + " hbm_gbs (burst; kernel timed alone over {} rotating layers)".format(len(tiles))}


def gemv_config1(ctx, stream, reps=8, copies=24):
    """BASELINE config 1 through the C-ABI: one 8192 x 2048 Q4 GEMV (synthetic Q4
    weights and N(0,1) x), timed back to back over `copies` packed copies
    of the matrix (226 MB, so no launch finds its 9.4 MB in L2)."""
    import torch
    from channel_b200 import _lib as L
    lib = L.load()
    M, K = 8192, 2048
    blocks = torch.empty(M * (K // 32) * 5, dtype=torch.int32, device="cuda")
    tb = lib.ch_q4_tile_bytes(M, K)
    tiles = torch.empty(copies * tb, dtype=torch.uint8, device="cuda")
    x = torch.randn(K, dtype=torch.float32, device="cuda", generator=torch.Generator("cuda").manual_seed(0))
    y = torch.empty(M, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    L.check(lib.ch_gen_q4_blocks(ctx.handle, blocks.data_ptr(), M, K, 1, 0.02))
    for c in range(copies):
        L.check(lib.ch_q4_pack(ctx.handle, blocks.data_ptr(), M, K, tiles.data_ptr() + c * tb))

    def call(i):
        L.check(lib.ch_gemv_q4(ctx.handle, tiles.data_ptr() + (i % copies) * tb, M, K, x.data_ptr(), y.data_ptr()))
    for i in range(copies):
        call(i)
    n = reps * copies
    k_ms = time_launches(ctx, stream, call, n)
    nbytes = M * K * 18 // 32 + K * 4 + M * 4
    peak, peak_kind = peaks()
    achieved = nbytes / (k_ms / 1000.0) / 1e9
    ctx.synchronize()
    del blocks, tiles, x, y
    return {"kernel": "gemv_kernel<Q4, STORE> (config 1: 8192 x 2048)", "achieved": achieved, "peak": peak,
            "unit": "GB/s", "frac": achieved / peak, "bytes_per_launch": nbytes, "us_per_launch": k_ms * 1000,
            "launches_timed": n, "peak_kind": peak_kind + " hbm_gbs (burst)"}


def config5(ctx, gm, cfg, stream, n_streams=64, n_tokens=128, lo=16, hi=2048, seed=4, rank=0, world=1):
    """BASELINE config 5 on the config-4 model: n_streams greedy streams, prompt lengths
    uniform in [lo, hi] and uniform token ids (seeded), n_tokens tokens each (the
    prefill's greedy token is the first), every stream with its own 4,096-slot ring KV.
    Prompts are prefilled stream by stream; then each decode step packs every stream
    (up to 64) into one ch_streams_decode call.  decode_tok_s = generated decode tokens
    / decode time (CUDA events on the library stream around all steps, the host ring
    bookkeeping between steps included); bytes_per_step = Q4 + Q8 weights once + every
    stream's K/V rows read.

    world > 1: stream-parallel replicas -- rank r holds a full copy of the weights and
    decodes streams [n r / world, n (r+1) / world) of the same seeded set, with no
    exchange between ranks; times are the max over ranks, tokens and bytes the sums."""
    import torch
    from channel_b200.streams import MultiStreamDecoder
    rng = np.random.default_rng(seed)
    all_lens = rng.integers(lo, hi + 1, n_streams)
    all_prompts = [rng.integers(0, cfg.vocab_size, int(n)).astype(np.uint32) for n in all_lens]
    mine = range(n_streams * rank // world, n_streams * (rank + 1) // world)
    lens = all_lens[mine.start:mine.stop]
    prompts = all_prompts[mine.start:mine.stop]
    n_mine = len(prompts)
    dec = MultiStreamDecoder(gm, cfg, n_mine, min(n_mine, 64))
    ctx.synchronize()
    t0 = time.time()
    longest = int(np.argmax(lens))
    for s, p in enumerate(prompts):
        if s == longest:  # NVTX ranges: what an ncu launch list filters on (--nvtx-include)
            torch.cuda.nvtx.range_push("config5_prefill_longest")
        dec.prefill(s, p)
        if s == longest:
            torch.cuda.nvtx.range_pop()
    ctx.synchronize()
    prefill_s = time.time() - t0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    kv_rows = 0  # K/V rows (all kv heads of one slot, per layer) the decode steps read
    n_full = sum(1 for full in cfg.layer_types[:cfg.num_hidden_layers] if full)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    e0.record(stream)
    while True:
        live = [s for s in range(n_mine) if len(dec.tokens[s]) < n_tokens]
        if not live:
            break
        for i in range(0, len(live), dec.max_batch):
            batch = live[i:i + dec.max_batch]
            for s in batch:
                c = dec.clock[s] + 1  # slots the step attends to
                kv_rows += n_full * min(c, 4096) + (cfg.num_hidden_layers - n_full) * min(c, cfg.sliding_window)
            mark = dec.steps == 1  # the second step (its graph already captured)
            if mark:
                torch.cuda.nvtx.range_push("config5_step")
            dec.step(batch)
            if mark:
                torch.cuda.nvtx.range_pop()
    e1.record(stream)
    e1.synchronize()
    decode_s = e0.elapsed_time(e1) / 1000.0
    steps = dec.steps
    tokens = n_streams * (n_tokens - 1)
    if world > 1:  # the slowest rank's times; every rank's K/V rows
        t = torch.tensor([decode_s, prefill_s, float(steps)], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        kv = torch.tensor([float(kv_rows)], device="cuda", dtype=torch.float64)
        dist.all_reduce(kv, op=dist.ReduceOp.SUM)
        decode_s, prefill_s, steps, kv_rows = float(t[0]), float(t[1]), int(t[2]), int(kv[0])
    weight_bytes = (cfg.num_hidden_layers * (cfg.hidden_size * (cfg.q_dim + 2 * cfg.kv_dim) + cfg.q_dim * cfg.hidden_size
                                             + 3 * cfg.hidden_size * cfg.intermediate_size) * 18 // 32
                    + cfg.vocab_size * cfg.hidden_size * 36 // 32)
    kv_bytes = kv_rows * 2 * cfg.kv_dim * 2
    step_bytes = world * weight_bytes + kv_bytes / steps  # every replica streams its weights
    peak, peak_kind = peaks()
    gbs = step_bytes / (decode_s / steps) / 1e9
    par = "single" if world == 1 else f"replicas{world} ({n_streams // world} streams per GPU, weights replicated, no exchange)"
    return {"workload": f"config5: {n_streams} streams, prompts U[{lo},{hi}] (seed {seed}), {n_tokens} greedy tokens each, "
                        "own 4096-slot ring KV per stream, one batched step for all streams",
            "parallelism": par,
            "prompt_tokens": int(all_lens.sum()), "prefill_s": prefill_s,
            "prefill_tok_s": float(all_lens.sum()) / prefill_s,
            "decode_steps": steps, "decode_s": decode_s, "decode_tok_s": tokens / decode_s,
            "ms_per_step": decode_s / steps * 1000, "bytes_per_step": step_bytes,
            "achieved_gbs": gbs, "peak_gbs": world * peak, "frac": gbs / (world * peak),
            "peak_kind": peak_kind + " hbm_gbs" + (f" x {world} GPUs" if world > 1 else ""),
            "tokens_head": [dec.tokens[s][:4] for s in range(min(2, n_mine))]}


def prefill_roofline(ctx, gm, cfg, stream, n_tok, layers=8, reps=2):
    """The prefill's Q4 GEMMs (tcgen05 kernel, CTA-pair M256xN256) on a 512-token
    batch: QKV, O, fused gate|up (+GELU*up) and down of `layers` consecutive layers,
    timed with CUDA events on the library stream.  achieved = algorithmic FLOPs
    (2 x tokens x weights) / time against the measured cuBLAS bf16 peak; the kernel
    issues three f16 MMAs per weight x activation product (exact split-scale
    weights, hi/lo activation), so its tensor-pipe work is 3x the algorithmic."""
    import torch
    from channel_b200 import _lib as L
    lib = L.load()
    H, I, qd = cfg.hidden_size, cfg.intermediate_size, cfg.q_dim
    xs = {k: torch.randn(n_tok, k, device="cuda", dtype=torch.float32) for k in {H, qd, I}}
    ybuf = torch.empty(n_tok * max(cfg.q_dim + 2 * cfg.kv_dim, I, H), device="cuda", dtype=torch.float32)
    torch.cuda.synchronize()
    kinds = ["qkv", "o", "gateup", "down"]

    def call(layer, which):
        tiles, rows, cols = gm.weight_tiles(layer, which)
        if which == 2:
            L.check(lib.ch_batch_fused_mlp_q4(ctx.handle, tiles, rows // 2, cols, xs[cols].data_ptr(), n_tok,
                                              ybuf.data_ptr()))
        else:
            L.check(lib.ch_batch_gemm_q4(ctx.handle, tiles, rows, cols, xs[cols].data_ptr(), n_tok, ybuf.data_ptr()))
        return 2.0 * n_tok * rows * cols

    per = {}
    for which in range(4):
        for l in range(layers):
            call(l, which)  # warm-up (and scratch sizing)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ctx.synchronize()
        e0.record(stream)
        flops = 0.0
        for _ in range(reps):
            for l in range(layers):
                flops += call(l, which)
        e1.record(stream)
        e1.synchronize()
        per[kinds[which]] = (flops, e0.elapsed_time(e1) / 1000.0)
    assert ctx.device_status() == 0
    flops = sum(f for f, _ in per.values())
    secs = sum(t for _, t in per.values())
    pk = ROOT / "MEASURED_PEAKS.json"
    peak, kind = (float(json.loads(pk.read_text())["bf16_tflops"]), "measured") if pk.exists() else (1590.0, "fallback")
    achieved = flops / secs / 1e12
    return {"bound": "tensor", "kernel": "batch_gemm_tc_kernel (tcgen05.mma.cta_group::2 kind::f16, M256 N256)",
            "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "mma_work_frac": 3 * achieved / peak, "tokens": n_tok,
            "per_gemm_tflops": {k: f / t / 1e12 for k, (f, t) in per.items()},
            "us_per_layer": secs / (reps * layers) * 1e6, "layers_timed": reps * layers,
            "peak_kind": kind + " bf16_tflops (cuBLAS burst); achieved = algorithmic 2*tokens*weights FLOPs"}


def nccl_exchange_floor(cfg, world, iters=20):
    """The collectives a tensor-parallel step would need if its two per-layer exchanges
    (the o and down partial sums) and the top-64 merge went through NCCL between kernel
    launches instead of the decode kernel's own NVLink peer stores: 2 x layers all-reduces
    of H floats and one all-gather of 64 candidates per token, captured in a CUDA graph
    and timed with events (the max over ranks).  A floor for that design: its kernels
    would also have to stop and restart around each collective."""
    import torch
    import torch.distributed as dist
    H = cfg.hidden_size
    bufs = [torch.zeros(H, device="cuda", dtype=torch.float32) for _ in range(2)]
    cand = torch.zeros(64, device="cuda", dtype=torch.int64)
    gath = torch.zeros(64 * world, device="cuda", dtype=torch.int64)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):  # warm NCCL up outside the capture
        for _ in range(3):
            dist.all_reduce(bufs[0])
            dist.all_gather_into_tensor(gath, cand)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for l in range(cfg.num_hidden_layers):
            dist.all_reduce(bufs[0])
            dist.all_reduce(bufs[1])
        dist.all_gather_into_tensor(gath, cand)
    g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        g.replay()
    e1.record()
    e1.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    del g  # the graph holds NCCL work: release it before the process group goes away
    torch.cuda.synchronize()
    return {"ms_per_token": ms, "collectives_per_token": 2 * cfg.num_hidden_layers + 1,
            "us_per_collective": ms * 1000 / (2 * cfg.num_hidden_layers + 1),
            "what": "2 x layers all-reduce of H f32 + 1 all-gather of 64 u64 per token, NCCL in a CUDA graph, "
                    "no compute: a floor for exchanging between kernel launches"}


def ours(args):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))

    from channel_b200 import DynamicRingBuffer, GpuContext, GpuModelContext, config_12b, gpu_dispatch_prefill_batch
    from channel_b200 import _lib as L
    from channel_b200.engine import gpu_dispatch_forward_token

    assert args.warmup >= 3, "at least 3 warm-up steps"
    cfg = config_12b(layers=args.layers)
    ctx = GpuContext.init(local)
    t0 = time.time()
    if world > 1:  # row-sharded tensor parallel: one token stream over all GPUs
        from channel_b200.engine import attach_tensor_parallel
        gm = GpuModelContext.synthetic_sharded(ctx, cfg, SEED, rank, world)
        attach_tensor_parallel(gm)
    else:
        gm = GpuModelContext.synthetic(ctx, cfg, SEED)
    build_s = time.time() - t0
    stream = torch.cuda.ExternalStream(ctx.stream)

    rng = np.random.default_rng(SEED)  # the same prompt on every rank
    prompt = rng.integers(0, cfg.vocab_size, PROMPT).astype(np.uint32)
    n_total = args.warmup + args.steps

    def fresh_prefill():
        gm.zero_state()
        if dist:
            dist.barrier()  # every rank's arrival counter is reset before any rank launches
        ring = DynamicRingBuffer(cfg.num_hidden_layers, 0)
        ring.setNumAnchors(min(PROMPT, 512))  # stream_handler.zig:67
        prev = ring.getPrefillPrevSlots(0, 0, PROMPT)
        slots = np.concatenate([prev, [ring.getSlotIndex(c) for c in range(PROMPT)]]).astype(np.uint32)
        for c in range(PROMPT):
            for l in range(cfg.num_hidden_layers):
                ring.activateSlot(l, c)
        torch.cuda.synchronize()
        t = time.time()
        cands = gpu_dispatch_prefill_batch(gm, prompt, None, slots, 0, len(prev))
        return ring, int(cands[0].id), time.time() - t  # host-synchronous: the call returns the top-64

    def step_lists(ring, clock):
        ring.activateSlot(0, clock)
        slot = ring.getSlotIndex(clock)
        return slot, ring.getActiveSlotsLayer(0, clock, False, cfg.sliding_window), \
            ring.getActiveSlotsLayer(0, clock, True, cfg.sliding_window)

    if args.kernel_only:
        r = gateup_roofline(ctx, gm, cfg, stream, reps=3)
        print(json.dumps({"kernel": "fused gate/up GEMV", **r}), flush=True)
        print(json.dumps(gemv_config1(ctx, stream)), flush=True)
        gm.deinit()
        ctx.deinit()
        return

    # ---- value: device-resident loop -------------------------------------------------
    # Every step builds its own ring lists on the device (ch_decode_run_ring: activate the
    # clock's slot, full and sliding lists), embeds the fed-back token and decodes: no
    # host work and no upload per token inside the timed region.
    from channel_b200 import DeviceRing
    ring, first, prefill_s = fresh_prefill()
    dring = DeviceRing(ctx)
    dring.upload(ring)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gm.decode_run_ring(dring, ring, first, PROMPT, args.warmup)
    warm_tokens = [int(t) for t in gm.decode_tokens(args.warmup)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        ev0.record(stream)
        gm.decode_run_ring(dring, ring, warm_tokens[-1], PROMPT + args.warmup, args.steps)
        ev1.record(stream)
        ev1.synchronize()
    ms = ev0.elapsed_time(ev1)
    torch.cuda.synchronize()
    tokens = warm_tokens + [int(t) for t in gm.decode_tokens(args.steps)]
    dring.deinit()
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    ms_per_step = ms / args.steps
    value = args.steps / (ms / 1000.0)  # one token stream, whatever the number of GPUs

    # ---- roofline: the dominant kernel is the persistent decode-step kernel (one launch
    # per token, >98% of the timed region; the tiny step_begin kernel is included)
    lib = L.load()
    H, I = cfg.hidden_size, cfg.intermediate_size
    peak, peak_kind = peaks()
    step_bytes = (cfg.num_hidden_layers * ((cfg.q_dim + 2 * cfg.kv_dim) * H + H * cfg.q_dim + 3 * I * H) * 18 // 32
                  + cfg.vocab_size * H * 36 // 32)
    kv_bytes = cfg.num_hidden_layers * 2 * 2 * cfg.kv_dim * (PROMPT + args.warmup + args.steps / 2)
    step_alg = (step_bytes + kv_bytes) / world  # this rank's shard of the weights and KV
    step_gbs = step_alg / (ms_per_step / 1000.0) / 1e9
    traffic = None
    tp = ROOT / "profiles" / "decode_step_traffic.json"
    if tp.exists():  # ncu DRAM bytes of one launch on a smaller case, scaled by algorithmic bytes
        t = json.loads(tp.read_text())
        traffic = t["dram_bytes"] * step_alg / t["algorithmic_bytes"]
    rl = {"bound": "hbm", "kernel": "decode_step_kernel (one greedy token: 48 layers, Q8 LM head, top-64)"
          + (f"; rank 0 of {world}, bytes = its shard" if world > 1 else ""),
          "achieved": step_gbs, "peak": peak, "unit": "GB/s", "frac": step_gbs / peak, "traffic": traffic,
          "bytes_per_launch": step_alg, "us_per_launch": ms_per_step * 1000, "launches_timed": args.steps,
          "peak_kind": peak_kind + " hbm_gbs (copy bandwidth); kernel timed inside the device loop"}
    # the Q4 GEMV on its own (metric's second part): fused gate/up, op-level kernel, rotating layers
    gemv_rl = gateup_roofline(ctx, gm, cfg, stream, reps=3) if world == 1 else None
    gemv_c1 = gemv_config1(ctx, stream) if world == 1 else None
    c5 = None
    if world == 1 and not args.no_config5 and cfg.num_hidden_layers == 48:
        c5 = config5(ctx, gm, cfg, stream, n_streams=args.config5_streams)
    elif world > 1 and not args.no_config5 and cfg.num_hidden_layers == 48:
        # stream-parallel replicas: a full copy of the weights on every rank beside its
        # tensor-parallel shard (which stays alive: its arena is mapped by the peers)
        gm5 = GpuModelContext.synthetic(ctx, cfg, SEED)
        c5 = config5(ctx, gm5, cfg, stream, n_streams=args.config5_streams, rank=rank, world=world)
        ctx.synchronize()
        gm5.deinit()
    # the batched prefill (one GPU): whole 512-token prompt, and its tensor-core GEMMs alone
    prefill_rl = None
    if world == 1:
        prefill_times = [fresh_prefill()[2] for _ in range(2)]
        prefill_rl = prefill_roofline(ctx, gm, cfg, stream, PROMPT, layers=min(8, cfg.num_hidden_layers))
        prefill_rl["prompt_s"] = min(prefill_times)
        prefill_rl["prompt_tok_s"] = PROMPT / min(prefill_times)

    nccl_floor = nccl_exchange_floor(cfg, world) if dist else None

    # ---- e2e: reference-facing call with host buffers ---------------------------------
    e2e = None
    if not args.no_e2e:
        emb_dev = torch.empty(cfg.vocab_size * H, dtype=torch.int16, device="cuda")
        L.check(lib.ch_gen_bf16(ctx.handle, emb_dev.data_ptr(), emb_dev.numel(),
                                lib.ch_tensor_seed(SEED, 0, 20), 0.0, 0.02))
        ctx.synchronize()
        table = emb_dev.cpu().numpy().view(np.uint16).reshape(cfg.vocab_size, H)
        del emb_dev
        scale = np.float32(math.sqrt(H))

        def embed(tok):
            return (table[tok].astype(np.uint32) << 16).view(np.float32) * scale

        ring, tok, _ = fresh_prefill()
        h2d = d2h = 0
        e_tokens = []
        for i in range(n_total):
            if i == args.warmup:
                ctx.synchronize()
                if dist:
                    dist.barrier()
                h2d = d2h = 0
                es0, es1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                es0.record(stream)
                tw = time.perf_counter()
            clock = PROMPT + i
            slot, act, sli = step_lists(ring, clock)
            x = embed(tok)
            tok, cands = gpu_dispatch_forward_token(gm, x, clock, slot, act, sli)
            e_tokens.append(tok)
            h2d += x.nbytes + 32 + 4 * (len(act) + len(sli))
            d2h += 64 * 8
        es1.record(stream)
        es1.synchronize()
        e_ms = es0.elapsed_time(es1)
        wall_ms = (time.perf_counter() - tw) * 1000
        e_ms = max(e_ms, wall_ms)
        if dist:
            t = torch.tensor([e_ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e_ms = float(t.item())
        e2e = {"value": args.steps / (e_ms / 1000.0), "unit": "tok/s",
               "h2d_bytes_per_step": h2d // args.steps, "d2h_bytes_per_step": d2h // args.steps,
               "ms_per_step": e_ms / args.steps,
               "tokens_match_device_loop": bool(list(e_tokens) == [int(t) for t in tokens])}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_sample(steps=4, warmup=1)
        cpu = {k: cpu[k] for k in ("value", "unit", "cores", "cpu_model", "kind", "sample", "timed_s")}

    launches_per_step = 3  # device ring lists + step_begin + the decode-step kernel
    if rank == 0:
        line = {
            "metric": "decode tok/s (12B-shape Q4) at 1/2/4/8 GPU; Q4 GEMV HBM GB/s vs peak",
            "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "q4/f16-mma/f32-acc", "data": "synthetic",
            "config": {**workload_config(cfg.num_hidden_layers, n_total),
                       "parallelism": f"tp{world} (row-sharded, in-kernel NVLink exchange)" if world > 1 else "single",
                       "l2": "per-step weight stream 7.2 GB > 126 MB L2 (no flush needed)"},
            "roofline": rl,
            "gemv_roofline": gemv_rl,
            "gemv_config1": gemv_c1,
            "config5": c5,
            "prefill_roofline": prefill_rl,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk.summary(),
            "setup_s": {"model_build": build_s, "prefill_512": prefill_s},
            "tokens_head": [int(t) for t in tokens[:8]],
            "tp_nccl_exchange_floor": nccl_floor,
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()  # no rank frees its arena while another may still run a kernel on it
    gm.deinit()
    ctx.deinit()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    a = parse()
    if a.impl == "reference":
        reference_arm(a)
    else:
        ours(a)
