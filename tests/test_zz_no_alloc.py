"""ch_gemv_q4_noalloc against ch_gemv_q4.

ch_gemv_q4_noalloc serves callers that may not allocate device memory (a host
runtime whose pool allocator owns the device's memory, a serving loop that
bans the device-wide synchronization of cudaFree, a binding that may only use
the buffers its caller hands over): its stream-K scratch is a static device
array inside the library instead of context memory.  These tests check that
it gives the ordinary entry point's results on consecutive calls (the shared
scratch must come back clean after each call) and that it refuses shapes the
array is not sized for.  This file is named to be collected last, so the
calls also run after everything else the suite has done on the device.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from channel_b200 import _lib as L
from tests.gpu_util import assert_close, call, dev, empty, host


def test_noalloc_rejects_shapes_beyond_its_scratch():
    lib = L.load()
    one = C.c_void_p(16)  # never dereferenced: the size check comes first
    assert lib.ch_gemv_q4_noalloc(one, 32784, 64, one, one, None, None) == L.CH_EINVAL
    assert "exceeds the static scratch" in lib.ch_last_error().decode()
    assert lib.ch_gemv_q4_noalloc(one, 16, 16448, one, one, None, None) == L.CH_EINVAL
    assert lib.ch_gemv_q4_noalloc(one, 24, 64, one, one, None, None) == L.CH_EINVAL
    assert lib.ch_gemv_q4_noalloc(None, 16, 64, one, one, None, None) == L.CH_EINVAL


@pytest.mark.gpu
def test_noalloc_matches_gemv_q4_on_consecutive_calls(ctx, oracle):
    lib = L.load()
    # a shape at the row limit, model shapes, then shapes with fewer row tiles than
    # CTAs (64 x 16384: 4 row tiles, 1024 x 8192: 64, 48 x 192: 3), where several CTAs
    # feed each row tile through the shared counters and partial slots: each call
    # reuses the counters the previous one left behind
    for M, K, seed in [(32768, 1024, 1), (3840, 15360, 2), (8192, 3840, 3), (64, 16384, 5), (1024, 8192, 6),
                       (48, 192, 4)]:
        W = oracle.gen_q4(M, K, oracle.tensor_seed(7, seed, 0))
        Wd = dev(W)
        tiles = empty(lib.ch_q4_tile_bytes(M, K), torch.uint8)
        call(lib.ch_q4_pack, ctx.handle, Wd.data_ptr(), M, K, tiles.data_ptr())
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        for rep in range(2):
            x = oracle.gen_f32(K, oracle.tensor_seed(7, seed, 100 + rep))
            xd, y_ref, y = dev(x), empty(M), empty(M)
            call(lib.ch_gemv_q4, ctx.handle, tiles.data_ptr(), M, K, xd.data_ptr(), y_ref.data_ptr())
            ctx.synchronize()
            call(lib.ch_gemv_q4_noalloc, tiles.data_ptr(), M, K, xd.data_ptr(), y.data_ptr(), status.data_ptr(),
                 ctx.stream)
            ctx.synchronize()
            assert_close(host(y), host(y_ref), what=f"noalloc {M}x{K} call {rep} vs ch_gemv_q4")
            assert_close(host(y), oracle.gemv_q4(W, x, M, K), what=f"noalloc {M}x{K} call {rep} vs oracle")
        assert int(status.item()) == 0
    # default stream and no status word
    M, K = 256, 2048
    W = oracle.gen_q4(M, K, oracle.tensor_seed(7, 9, 0))
    Wd = dev(W)
    tiles = empty(lib.ch_q4_tile_bytes(M, K), torch.uint8)
    call(lib.ch_q4_pack, ctx.handle, Wd.data_ptr(), M, K, tiles.data_ptr())
    x = oracle.gen_f32(K, oracle.tensor_seed(7, 9, 100))
    xd, y = dev(x), empty(M)
    ctx.synchronize()
    call(lib.ch_gemv_q4_noalloc, tiles.data_ptr(), M, K, xd.data_ptr(), y.data_ptr(), None, None)
    torch.cuda.synchronize()
    assert_close(host(y), oracle.gemv_q4(W, x, M, K), what="noalloc on the default stream vs oracle")


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs a second GPU")
def test_noalloc_and_gemv_on_a_second_device(ctx, oracle):
    """Both GEMV entry points on device 1 after device 0 has run them (the session
    context): the dynamic shared-memory attribute (147 KB) and the no-alloc scratch are
    per device, so the first launch on the second device must set up its own."""
    from channel_b200 import GpuContext
    lib = L.load()
    M, K = 3840, 15360
    W = oracle.gen_q4(M, K, oracle.tensor_seed(7, 11, 0))
    with torch.cuda.device(1):
        c1 = GpuContext.init(1)
        try:
            tiles = empty(lib.ch_q4_tile_bytes(M, K), torch.uint8)
            Wd = dev(W)
            call(lib.ch_q4_pack, c1.handle, Wd.data_ptr(), M, K, tiles.data_ptr())
            status = torch.zeros(1, dtype=torch.int32, device="cuda")
            for rep in range(2):
                x = oracle.gen_f32(K, oracle.tensor_seed(7, 11, 100 + rep))
                ref = oracle.gemv_q4(W, x, M, K)
                xd, y1, y2 = dev(x), empty(M), empty(M)
                torch.cuda.synchronize()
                call(lib.ch_gemv_q4, c1.handle, tiles.data_ptr(), M, K, xd.data_ptr(), y1.data_ptr())
                c1.synchronize()
                call(lib.ch_gemv_q4_noalloc, tiles.data_ptr(), M, K, xd.data_ptr(), y2.data_ptr(), status.data_ptr(),
                     c1.stream)
                c1.synchronize()
                assert_close(host(y1), ref, what=f"ch_gemv_q4 on device 1, call {rep}")
                assert_close(host(y2), ref, what=f"noalloc on device 1, call {rep}")
            assert int(status.item()) == 0
            assert c1.device_status() == 0
        finally:
            c1.synchronize()
            c1.deinit()
