"""Prefill GEMM timings (a measurement and profiling aid).

Times the tensor-core prefill GEMMs (ch_batch_gemm_q4 / ch_batch_fused_mlp_q4,
tcgen05 CTA-pair kernel) against the legacy mma.sync kernels
(ch_batch_gemm_q4_mma / ch_batch_fused_mlp_q4_mma) on the 12B and config-3 layer
shapes, with synthetic Q4 weights from the device generator and CUDA events on
the library's stream.  TF/s are algorithmic (2 x tokens x weights).

  python bench_gemm.py [--tokens 512]
  python bench_gemm.py --only gateup12b --launches 3   # e.g. under ncu -k regex:batch_gemm_tc
"""
from __future__ import annotations

import argparse
import sys

SHAPES = [  # name, output rows, cols (K), fused gate|up
    ("qkv12b", 8192, 3840, False), ("o12b", 3840, 4096, False), ("gateup12b", 15360, 3840, True),
    ("down12b", 3840, 15360, False), ("qkv_c3", 2560, 2048, False), ("gateup_c3", 8192, 2048, True),
    ("down_c3", 2048, 8192, False)]


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=512)
    ap.add_argument("--only", default=None, help="one shape name; with --launches, no timing")
    ap.add_argument("--launches", type=int, default=0, help="just run the tensor-core GEMM this many times")
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()

    import torch

    from channel_b200 import _lib as L
    from channel_b200 import GpuContext
    lib = L.load()
    ctx = GpuContext.init(0)
    stream = torch.cuda.ExternalStream(ctx.stream)
    N = args.tokens
    keep = []
    for name, M, K, gate in SHAPES:
        if args.only and name != args.only:
            continue
        rows = 2 * M if gate else M
        tiles = torch.empty(lib.ch_q4_tile_bytes(rows, K), dtype=torch.uint8, device="cuda")
        blocks = torch.empty(rows * (K // 32) * 5, dtype=torch.int32, device="cuda")
        X = torch.randn(N, K, device="cuda")
        Y = torch.empty(N * M, device="cuda")
        torch.cuda.synchronize()  # X is written on torch's stream, the library works on its own
        L.check(lib.ch_gen_q4_blocks(ctx.handle, blocks.data_ptr(), rows, K, 7, 0.02))
        if gate:
            half = blocks.data_ptr() + M * (K // 32) * 5 * 4
            L.check(lib.ch_q4_pack_gateup(ctx.handle, blocks.data_ptr(), half, M, K, tiles.data_ptr()))
        else:
            L.check(lib.ch_q4_pack(ctx.handle, blocks.data_ptr(), M, K, tiles.data_ptr()))
        base = "ch_batch_fused_mlp_q4" if gate else "ch_batch_gemm_q4"
        if args.launches:
            for _ in range(args.launches):
                L.check(getattr(lib, base)(ctx.handle, tiles.data_ptr(), M, K, X.data_ptr(), N, Y.data_ptr()))
            ctx.synchronize()
            keep.append((tiles, blocks, X, Y))
            continue
        flops = 2.0 * N * rows * K
        res = {}
        for impl in ("", "_mma"):
            fn = getattr(lib, base + impl)
            for _ in range(3):
                L.check(fn(ctx.handle, tiles.data_ptr(), M, K, X.data_ptr(), N, Y.data_ptr()))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.iters):
                L.check(fn(ctx.handle, tiles.data_ptr(), M, K, X.data_ptr(), N, Y.data_ptr()))
            e1.record(stream)
            e1.synchronize()
            res[impl] = e0.elapsed_time(e1) / args.iters / 1000.0
        ctx.synchronize()
        keep.append((tiles, blocks, X, Y))  # freed only after the library's stream is idle
        print(f"{name:10s} tokens {N} rows {rows} K {K}: tcgen05 {res[''] * 1e6:8.1f} us "
              f"({flops / res[''] / 1e12:6.1f} TF/s)  mma.sync {res['_mma'] * 1e6:8.1f} us "
              f"({flops / res['_mma'] / 1e12:6.1f} TF/s)", flush=True)
    status = ctx.device_status()
    print("device status", status)
    ctx.deinit()
    return 0 if status == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
