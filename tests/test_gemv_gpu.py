"""GPU parity of the decode matvec family against the oracle (gemv_q4.wgsl,
fused_mlp_q4.wgsl, gemv_q8.wgsl), the repack, and the device generator."""
import numpy as np
import pytest
import torch

from channel_b200 import _lib as L
from tests.gpu_util import assert_close, call, dev, empty, host

pytestmark = pytest.mark.gpu


def test_device_generator_matches_oracle(ctx, oracle):
    lib = L.load()
    for rows, cols, ts in [(17, 64, 5), (256, 3840, oracle.tensor_seed(3, 7, 0))]:
        ref = oracle.gen_q4(rows, cols, ts)
        d = empty(ref.size, torch.int32)
        call(lib.ch_gen_q4_blocks, ctx.handle, d.data_ptr(), rows, cols, ts, 0.02)
        ctx.synchronize()
        assert np.array_equal(host(d, np.uint32).reshape(ref.shape), ref)
    n = 3 * 3840 + 7
    ref = oracle.gen_bf16(n, 77, 0.0, 0.02)
    d = empty(n, torch.int16)
    call(lib.ch_gen_bf16, ctx.handle, d.data_ptr(), n, 77, 0.0, 0.02)
    ctx.synchronize()
    assert np.array_equal(host(d, np.uint16), ref)
    ref = oracle.gen_bf16(n, 78, 1.0, 0.02)
    call(lib.ch_gen_bf16, ctx.handle, d.data_ptr(), n, 78, 1.0, 0.02)
    ctx.synchronize()
    assert np.array_equal(host(d, np.uint16), ref)


@pytest.mark.parametrize("mode", [4, 8])
def test_device_quantizer_matches_oracle(ctx, oracle, mode):
    lib = L.load()
    rows, cols = 64, 3840
    src = oracle.gen_bf16(rows * cols, 9, 0.0, 0.02)
    ref = oracle.quantize_matrix(src, rows, cols, mode)
    d = empty(ref.size, torch.int32)
    fn = lib.ch_quantize_q8_rows if mode == 8 else lib.ch_quantize_q4_rows
    srcd = dev(src)
    call(fn, ctx.handle, srcd.data_ptr(), rows, cols, d.data_ptr())
    ctx.synchronize()
    assert np.array_equal(host(d, np.uint32).reshape(ref.shape), ref)


# config 1 (8192 x 2048, seed 0) plus model shapes and small / odd shapes
SHAPES = [(8192, 2048), (16, 64), (48, 192), (8192, 3840), (3840, 4096), (3840, 15360), (256, 2048), (4096, 64)]


@pytest.mark.parametrize("M,K", SHAPES)
def test_gemv_q4_parity(ctx, oracle, M, K):
    lib = L.load()
    W = oracle.gen_q4(M, K, oracle.tensor_seed(0, 0, 0))
    x = oracle.gen_f32(K, oracle.tensor_seed(0, 0, 100))
    ref = oracle.gemv_q4(W, x, M, K)
    tiles = empty(lib.ch_q4_tile_bytes(M, K), torch.uint8)
    xd, yd, Wd = dev(x), empty(M), dev(W)
    call(lib.ch_q4_pack, ctx.handle, Wd.data_ptr(), M, K, tiles.data_ptr())
    for _ in range(2):  # second launch checks the stream-K counters were reset
        yd.fill_(float("nan"))
        call(lib.ch_gemv_q4, ctx.handle, tiles.data_ptr(), M, K, xd.data_ptr(), yd.data_ptr())
        ctx.synchronize()
        e = assert_close(host(yd), ref, what=f"gemv_q4 {M}x{K}")
        assert e < 1e-5  # hi/lo split keeps fp32 accuracy
    assert ctx.device_status() == 0


@pytest.mark.parametrize("M,K", [(15360, 3840), (8192, 2048), (8, 64), (1920, 3840)])
def test_fused_mlp_q4_parity(ctx, oracle, M, K):
    lib = L.load()
    Wg = oracle.gen_q4(M, K, oracle.tensor_seed(2, 0, 4))
    Wu = oracle.gen_q4(M, K, oracle.tensor_seed(2, 0, 5))
    x = oracle.gen_f32(K, 5)
    ref = oracle.fused_mlp_q4(Wg, Wu, x, M, K)
    tiles = empty(lib.ch_q4_tile_bytes(2 * M, K), torch.uint8)
    yd, Wgd, Wud, xd = empty(M), dev(Wg), dev(Wu), dev(x)
    call(lib.ch_q4_pack_gateup, ctx.handle, Wgd.data_ptr(), Wud.data_ptr(), M, K, tiles.data_ptr())
    call(lib.ch_fused_mlp_q4, ctx.handle, tiles.data_ptr(), M, K, xd.data_ptr(), yd.data_ptr())
    ctx.synchronize()
    assert_close(host(yd), ref, what="fused_mlp_q4")


@pytest.mark.parametrize("M,K", [(262144, 3840), (4096, 512), (16, 32)])
def test_gemv_q8_parity(ctx, oracle, M, K):
    lib = L.load()
    emb = oracle.gen_bf16(M * K, 21, 0.0, 0.02)
    W = oracle.quantize_matrix(emb, M, K, 8)
    x = oracle.gen_f32(K, 6)
    ref = oracle.gemv_q8(W, x, M, K)
    tiles = empty(lib.ch_q8_tile_bytes(M, K), torch.uint8)
    yd, Wd, xd = empty(M), dev(W), dev(x)
    call(lib.ch_q8_pack, ctx.handle, Wd.data_ptr(), M, K, tiles.data_ptr())
    call(lib.ch_gemv_q8, ctx.handle, tiles.data_ptr(), M, K, xd.data_ptr(), yd.data_ptr())
    ctx.synchronize()
    assert_close(host(yd), ref, what="gemv_q8")


def test_gemv_rejects_bad_shapes(ctx):
    lib = L.load()
    assert lib.ch_gemv_q4(ctx.handle, 1, 17, 64, 1, 1) == L.CH_EINVAL
    assert lib.ch_gemv_q4(ctx.handle, 1, 16, 96, 1, 1) == L.CH_EINVAL
    assert lib.ch_q8_pack(ctx.handle, 1, 16, 48, 1) == L.CH_EINVAL
