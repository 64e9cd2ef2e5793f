"""GPU top-64 (topk_pass1/2.wgsl + greedy candidates[0]) against the oracle:
ids bit-exact with the (value desc, lowest index) rule, softcapped values close."""
import numpy as np
import pytest
import torch

from channel_b200 import _lib as L
from tests.gpu_util import call, dev, empty, host

pytestmark = pytest.mark.gpu


def run(ctx, oracle, logits):
    lib = L.load()
    ids, vals, lg = empty(64, torch.int32), empty(64), dev(logits)
    call(lib.ch_topk64, ctx.handle, lg.data_ptr(), logits.size, ids.data_ptr(), vals.data_ptr())
    ctx.synchronize()
    rid, rvals = oracle.topk64(logits)
    return host(ids, np.uint32), host(vals), rid, rvals


@pytest.mark.parametrize("V", [262144, 100000, 2048, 100, 64])
def test_random_logits(ctx, oracle, V):
    lg = (np.random.default_rng(V).standard_normal(V) * 3).astype(np.float32)
    ids, vals, rid, rvals = run(ctx, oracle, lg)
    assert np.array_equal(ids, rid)
    assert np.allclose(vals, rvals, rtol=2e-6, atol=1e-6)
    assert ids[0] == int(np.argmax(lg))


def test_ties_lowest_index_first(ctx, oracle):
    lg = np.zeros(262144, np.float32)
    lg[[200000, 7, 150000, 9]] = 2.0
    lg[123456] = 5.0
    ids, vals, rid, rvals = run(ctx, oracle, lg)
    assert np.array_equal(ids, rid)
    assert list(ids[:5]) == [123456, 7, 9, 150000, 200000]
    assert list(ids[5:9]) == [0, 1, 2, 3]


def test_saturating_softcap_ties(ctx, oracle):
    # very large logits all softcap to 30.0 -> ordering falls back to index
    lg = np.full(5000, -1.0, np.float32)
    lg[[4000, 10, 2500]] = [1e4, 2e4, 3e4]
    ids, vals, rid, rvals = run(ctx, oracle, lg)
    assert np.array_equal(ids, rid)
    assert list(ids[:3]) == [10, 2500, 4000] and np.all(vals[:3] == 30.0)


def test_fewer_than_64(ctx, oracle):
    lg = np.arange(20, dtype=np.float32)
    ids, vals, rid, rvals = run(ctx, oracle, lg)
    assert list(ids[:20]) == list(range(19, -1, -1))
    assert np.array_equal(ids, rid)
