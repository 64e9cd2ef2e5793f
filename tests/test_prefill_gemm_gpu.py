"""GPU parity of the tcgen05 prefill GEMMs (batch_gemm_q4.wgsl,
batch_fused_mlp_q4.wgsl) against the oracle, on config 3's shapes, ragged token
counts (partial 128-token tiles), row counts that are not a multiple of 128 and
the 12B shapes (those against the oracle on a subset of tokens and against the
legacy mma.sync kernel on all of them).  17 to 64 tokens run the skinny tcgen05
kernel of the multi-stream decode step (tokens on the MMA's M side, 256 weight rows
per CTA, split K): those shapes include row counts that are not a multiple of 256
and K loops of one to sixty k tiles per split."""
import numpy as np
import pytest
import torch

from channel_b200 import _lib as L
from tests.gpu_util import assert_close, call, dev, empty, host

pytestmark = pytest.mark.gpu

# the weights enter exactly (q-8 in f16) and the activation as an f16 hi + lo pair,
# so the GEMM keeps fp32 accuracy well inside the 1e-3 bar
FP32_FAITHFUL = 1e-5


def _pack(lib, ctx, W, M, K):
    tiles = empty(lib.ch_q4_tile_bytes(M, K), torch.uint8)
    Wd = dev(W)
    call(lib.ch_q4_pack, ctx.handle, Wd.data_ptr(), M, K, tiles.data_ptr())
    return tiles


def _pack_gateup(lib, ctx, Wg, Wu, M, K):
    tiles = empty(lib.ch_q4_tile_bytes(2 * M, K), torch.uint8)
    Wgd, Wud = dev(Wg), dev(Wu)
    call(lib.ch_q4_pack_gateup, ctx.handle, Wgd.data_ptr(), Wud.data_ptr(), M, K, tiles.data_ptr())
    return tiles


# (N tokens, M rows, K): config 3's QKV / O / down, ragged and small shapes
GEMM_SHAPES = [(512, 2560, 2048), (512, 2048, 2048), (512, 2048, 8192), (1, 16, 64), (24, 48, 192), (130, 272, 2048),
               (300, 2560, 128), (1024, 128, 64), (17, 272, 2048), (64, 2560, 2048), (40, 4112, 512), (64, 16, 64)]


@pytest.mark.parametrize("N,M,K", GEMM_SHAPES)
def test_batch_gemm_q4_parity(ctx, oracle, N, M, K):
    lib = L.load()
    W = oracle.gen_q4(M, K, oracle.tensor_seed(2, 0, 0))
    X = oracle.gen_f32(N * K, oracle.tensor_seed(2, 0, 100)).reshape(N, K)
    ref = oracle.batch_gemm_q4(W, X, N, M, K)
    tiles = _pack(lib, ctx, W, M, K)
    xd, yd = dev(X), empty(N * M)
    for _ in range(2):  # a second call on the same scratch
        yd.fill_(float("nan"))
        call(lib.ch_batch_gemm_q4, ctx.handle, tiles.data_ptr(), M, K, xd.data_ptr(), N, yd.data_ptr())
        ctx.synchronize()
        e = assert_close(host(yd).reshape(N, M), ref, what=f"batch_gemm_q4 {N}x{M}x{K}")
        assert e < FP32_FAITHFUL
    assert ctx.device_status() == 0


# (N, I, K): config 3's gate|up, ragged and small
MLP_SHAPES = [(512, 8192, 2048), (24, 8, 64), (130, 40, 192), (200, 1920, 3840), (64, 1920, 3840), (33, 40, 192)]


@pytest.mark.parametrize("N,M,K", MLP_SHAPES)
def test_batch_fused_mlp_q4_parity(ctx, oracle, N, M, K):
    lib = L.load()
    Wg = oracle.gen_q4(M, K, oracle.tensor_seed(2, 0, 4))
    Wu = oracle.gen_q4(M, K, oracle.tensor_seed(2, 0, 5))
    X = oracle.gen_f32(N * K, 11).reshape(N, K)
    ref = oracle.batch_fused_mlp_q4(Wg, Wu, X, N, M, K)
    tiles = _pack_gateup(lib, ctx, Wg, Wu, M, K)
    xd, yd = dev(X), empty(N * M)
    yd.fill_(float("nan"))
    call(lib.ch_batch_fused_mlp_q4, ctx.handle, tiles.data_ptr(), M, K, xd.data_ptr(), N, yd.data_ptr())
    ctx.synchronize()
    e = assert_close(host(yd).reshape(N, M), ref, what=f"batch_fused_mlp_q4 {N}x{M}x{K}")
    assert e < FP32_FAITHFUL
    assert ctx.device_status() == 0


def test_batch_fused_mlp_q4_fresh_context(oracle):
    """The fused gate|up GEMM as the first call on a new context: the entry point
    sizes the context's scratch itself (the other tests share one context whose
    scratch earlier GEMMs already grew)."""
    from channel_b200 import GpuContext
    lib = L.load()
    N, M, K = 300, 520, 512
    Wg = oracle.gen_q4(M, K, oracle.tensor_seed(2, 1, 4))
    Wu = oracle.gen_q4(M, K, oracle.tensor_seed(2, 1, 5))
    X = oracle.gen_f32(N * K, 12).reshape(N, K)
    ref = oracle.batch_fused_mlp_q4(Wg, Wu, X, N, M, K)
    c = GpuContext.init(0)
    try:
        tiles = _pack_gateup(lib, c, Wg, Wu, M, K)
        xd, yd = dev(X), empty(N * M)
        yd.fill_(float("nan"))
        torch.cuda.synchronize()
        call(lib.ch_batch_fused_mlp_q4, c.handle, tiles.data_ptr(), M, K, xd.data_ptr(), N, yd.data_ptr())
        c.synchronize()
        e = assert_close(host(yd).reshape(N, M), ref, what=f"batch_fused_mlp_q4 fresh {N}x{M}x{K}")
        assert e < FP32_FAITHFUL
        assert c.device_status() == 0
    finally:
        c.synchronize()
        c.deinit()


@pytest.mark.parametrize("N", [512, 64, 17])
@pytest.mark.parametrize("kind,M,K", [("gemm", 8192, 3840), ("gemm", 3840, 4096), ("gemm", 3840, 15360),
                                      ("mlp", 15360, 3840)])
def test_12b_shapes_against_oracle_and_mma_path(ctx, oracle, kind, M, K, N):
    """512 tokens (the prefill kernel) and 64 / 17 (the skinny kernel of the
    multi-stream step) at the 12B shapes: every output against the oracle (seconds of
    CPU at these sizes) and against the mma.sync kernel."""
    lib = L.load()
    X = oracle.gen_f32(N * K, 13).reshape(N, K)
    sel = np.arange(N)
    Xs = X
    if kind == "gemm":
        W = oracle.gen_q4(M, K, oracle.tensor_seed(3, 0, 1))
        tiles = _pack(lib, ctx, W, M, K)
        fn, fn_mma, rows_out = lib.ch_batch_gemm_q4, lib.ch_batch_gemm_q4_mma, M
        ref = oracle.batch_gemm_q4(W, Xs, len(sel), M, K)
    else:
        Wg = oracle.gen_q4(M, K, oracle.tensor_seed(3, 0, 4))
        Wu = oracle.gen_q4(M, K, oracle.tensor_seed(3, 0, 5))
        tiles = _pack_gateup(lib, ctx, Wg, Wu, M, K)
        fn, fn_mma, rows_out = lib.ch_batch_fused_mlp_q4, lib.ch_batch_fused_mlp_q4_mma, M
        ref = oracle.batch_fused_mlp_q4(Wg, Wu, Xs, len(sel), M, K)
    xd, y, y2 = dev(X), empty(N * rows_out), empty(N * rows_out)
    call(fn, ctx.handle, tiles.data_ptr(), M, K, xd.data_ptr(), N, y.data_ptr())
    call(fn_mma, ctx.handle, tiles.data_ptr(), M, K, xd.data_ptr(), N, y2.data_ptr())
    ctx.synchronize()
    Y = host(y).reshape(N, rows_out)
    assert assert_close(Y[sel], ref, what=f"{kind} {M}x{K} vs oracle ({len(sel)} tokens)") < FP32_FAITHFUL
    assert assert_close(Y, host(y2).reshape(N, rows_out), what=f"{kind} {M}x{K} vs mma.sync") < FP32_FAITHFUL
    assert ctx.device_status() == 0


def test_batch_gemm_rejects_bad_shapes(ctx):
    lib = L.load()
    assert lib.ch_batch_gemm_q4(ctx.handle, 16, 24, 64, 16, 4, 16) == L.CH_EINVAL  # rows % 16
    assert lib.ch_batch_gemm_q4(ctx.handle, 16, 32, 96, 16, 4, 16) == L.CH_EINVAL  # cols % 64
