"""GPU parity of fused qk-norm + RoPE + KV write + decode attention
(qkv_rope.wgsl + decode_attn.wgsl) against the oracle; config 2 and edge cases."""
import numpy as np
import pytest
import torch

from channel_b200 import _lib as L
from tests.gpu_util import assert_close, call, dev, empty, host

pytestmark = pytest.mark.gpu


def run_case(ctx, oracle, nq, nkv, slots, clock, slot, theta=1e4, scale=1 / 16, seed=1, rot=256):
    D = 256
    rng = np.random.default_rng(seed)
    kc = rng.standard_normal((4096, nkv * D)).astype(np.float16).view(np.uint16)
    vc = rng.standard_normal((4096, nkv * D)).astype(np.float16).view(np.uint16)
    q = rng.standard_normal(nq * D).astype(np.float32)
    k = rng.standard_normal(nkv * D).astype(np.float32)
    v = rng.standard_normal(nkv * D).astype(np.float32)
    qn = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    kn = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    slots = np.asarray(slots, np.uint32)
    # oracle: qkv_rope writes the new K/V (f16) into the cache, then attention
    kc_ref, vc_ref = kc.copy(), vc.copy()
    q_rot = oracle.qkv_rope(q, k, v, qn, kn, kc_ref, vc_ref, nq, nkv, D, rot, theta, 1e-6, clock, slot)
    ref = oracle.decode_attn(q_rot, kc_ref, vc_ref, slots, nq, nkv, D, scale)
    # device
    lib = L.load()
    kcd, vcd = dev(kc), dev(vc)
    qkv = dev(np.concatenate([q, k, v]))
    out = empty(nq * D)
    sd = dev(slots) if slots.size else empty(1, torch.int32)
    qnd, knd = dev(qn), dev(kn)
    call(lib.ch_decode_attention, ctx.handle, qkv.data_ptr(), qnd.data_ptr(), knd.data_ptr(), kcd.data_ptr(),
         vcd.data_ptr(), sd.data_ptr(), slots.size, clock, slot, nq, nkv, D, rot, theta, 1e-6, scale, out.data_ptr())
    ctx.synchronize()
    got_k = host(kcd, np.uint16).reshape(4096, -1)
    got_v = host(vcd, np.uint16).reshape(4096, -1)
    # cache: only `slot` changed, and it holds the normed/roped K and unit-normed V (f16)
    mask = np.ones(4096, bool)
    mask[slot] = False
    assert np.array_equal(got_k[mask], kc_ref.reshape(4096, -1)[mask])
    assert np.array_equal(got_v[mask], vc_ref.reshape(4096, -1)[mask])
    for got, want in ((got_k[slot], kc_ref.reshape(4096, -1)[slot]), (got_v[slot], vc_ref.reshape(4096, -1)[slot])):
        a = got.view(np.float16).astype(np.float64)
        b = want.view(np.float16).astype(np.float64)
        assert np.max(np.abs(a - b) / (np.abs(b) + 1e-3)) < 2e-3  # within 2 f16 ulps
    if slots.size:
        assert_close(host(out), ref, what="decode_attn")
    else:
        assert np.all(host(out) == 0)
    assert ctx.device_status() == 0


def test_config2_wrapped_ring(ctx, oracle):
    # 16 q / 8 kv heads, D 256, 3,000 filled slots starting at 1,500 (wraps past 4095),
    # current position 2,999 -> its K/V overwrite slot (1500 + 2999) % 4096 = 403
    slots = [(1500 + i) % 4096 for i in range(3000)]
    run_case(ctx, oracle, 16, 8, slots, clock=2999, slot=slots[-1])


@pytest.mark.parametrize("nq,nkv", [(8, 8), (16, 4), (8, 1), (32, 8)])
def test_gqa_ratios(ctx, oracle, nq, nkv):
    slots = list(range(0, 700))
    run_case(ctx, oracle, nq, nkv, slots, clock=699, slot=699, theta=1e6, scale=1.0, seed=nq + nkv)


def test_single_slot_and_full_ring(ctx, oracle):
    run_case(ctx, oracle, 16, 8, [5], clock=5, slot=5)
    run_case(ctx, oracle, 16, 8, list(range(4096)), clock=5000, slot=1234, seed=3)


def test_empty_list_and_partial_rotary(ctx, oracle):
    run_case(ctx, oracle, 16, 8, [], clock=0, slot=0)
    run_case(ctx, oracle, 16, 8, list(range(37)), clock=36, slot=36, rot=128, seed=4)


def test_current_slot_not_in_list(ctx, oracle):
    # the new K/V are still written; attention only reads the listed slots
    run_case(ctx, oracle, 16, 8, list(range(10, 90)), clock=200, slot=3)


def test_rejects_out_of_range(ctx):
    lib = L.load()
    assert lib.ch_decode_attention(ctx.handle, 1, 1, 1, 1, 1, 1, 10, 0, 4096, 16, 8, 256, 256, 1e4, 1e-6, 1.0, 1) == L.CH_EINVAL
    assert lib.ch_decode_attention(ctx.handle, 1, 1, 1, 1, 1, 1, 4097, 0, 0, 16, 8, 256, 256, 1e4, 1e-6, 1.0, 1) == L.CH_EINVAL
    assert lib.ch_decode_attention(ctx.handle, 1, 1, 1, 1, 1, 1, 1, 0, 0, 16, 8, 128, 128, 1e4, 1e-6, 1.0, 1) == L.CH_EINVAL
