"""GPU parity of the row norms (batch_rmsnorm.wgsl / batch_add_rmsnorm.wgsl, the
prefill and multi-stream steps' norms) against the oracle: the register path
(H % 4 == 0, H <= 4096), the strided path (other H), one to 1024 rows, in place
(y == x) and the residual add's write-back of x."""
import numpy as np
import pytest

from channel_b200 import _lib as L
from tests.gpu_util import assert_close, call, dev, empty, host

pytestmark = pytest.mark.gpu

EPS = 1e-6
# the oracle sums the squares in order, the kernels per thread then across the block:
# the two sums differ by a few ulps of a 4096-term sum
TOL = 1e-5
SHAPES = [(1, 3840), (64, 3840), (7, 2048), (3, 4096), (5, 4100), (9, 130), (1024, 512), (2, 4)]


def _inputs(n, h, seed):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((n, h)) * 3).astype(np.float32)
    r = rng.standard_normal((n, h)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(h)).astype(np.float32)
    return x, r, w


@pytest.mark.parametrize("n,h", SHAPES)
def test_rmsnorm_rows(ctx, oracle, n, h):
    lib, ol = L.load(), oracle.lib()
    x, _, w = _inputs(n, h, 1 + n + h)
    ref = np.empty_like(x)
    ol.or_batch_rmsnorm(oracle.p(ref, oracle.f32), oracle.p(x, oracle.f32), oracle.p(w, oracle.f32), n, h, EPS)
    xd, wd, yd = dev(x), dev(w), empty(n * h)
    call(lib.ch_rmsnorm, ctx.handle, xd.data_ptr(), wd.data_ptr(), yd.data_ptr(), n, h, EPS)
    ctx.synchronize()
    assert assert_close(host(yd).reshape(n, h), ref, what=f"rmsnorm {n}x{h}") < TOL
    # in place, as the post-attention / post-FFN norms run
    call(lib.ch_rmsnorm, ctx.handle, xd.data_ptr(), wd.data_ptr(), xd.data_ptr(), n, h, EPS)
    ctx.synchronize()
    assert assert_close(host(xd).reshape(n, h), ref, what=f"rmsnorm in place {n}x{h}") < TOL


@pytest.mark.parametrize("n,h", SHAPES)
def test_add_rmsnorm_rows(ctx, oracle, n, h):
    lib, ol = L.load(), oracle.lib()
    x, r, w = _inputs(n, h, 2 + n + h)
    scalar = 0.75
    xo, ref = x.copy(), np.empty_like(x)
    ol.or_batch_add_rmsnorm(oracle.p(xo, oracle.f32), oracle.p(r, oracle.f32), oracle.p(w, oracle.f32),
                            oracle.p(ref, oracle.f32), n, h, EPS, scalar)
    xd, rd, wd, yd = dev(x), dev(r), dev(w), empty(n * h)
    call(lib.ch_add_rmsnorm, ctx.handle, xd.data_ptr(), rd.data_ptr(), wd.data_ptr(), yd.data_ptr(), n, h, EPS, scalar)
    ctx.synchronize()
    np.testing.assert_array_equal(host(xd).reshape(n, h), xo)  # (x + r) * scalar: one rounding each, exact
    assert assert_close(host(yd).reshape(n, h), ref, what=f"add_rmsnorm {n}x{h}") < TOL
    assert ctx.device_status() == 0
