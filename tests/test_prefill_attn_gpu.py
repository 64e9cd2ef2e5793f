"""batch_causal_attn (shaders/batch_causal_attn.wgsl:25-223) on its own, through
ch_batch_causal_attention, against the oracle's restatement (or_batch_causal_attn):
BASELINE config 3's shape (512 tokens, 8 q heads on 1 kv head, no previous slots),
chunks that attend to earlier slots (prefix), the 1,024-slot sliding window of
sliding layers (:52-53) starting inside and across a chunk, ragged token counts,
scattered physical slots, and every GQA grouping (pairs of q heads per kv head run
on the tensor-core kernel, single heads on the CUDA-core one).  The tensor cores'
f32 sums are not rounded like the shader's per-slot recurrence: 1e-3 relative."""
import numpy as np
import pytest

from channel_b200 import _lib as L
from tests.gpu_util import assert_close, call, dev, empty, host

pytestmark = pytest.mark.gpu
D = 256


@pytest.mark.parametrize("N,num_prev,nq,nkv,sliding,scatter", [
    (512, 0, 8, 1, False, False),
    (64, 100, 8, 1, False, True),      # a chunk after 100 earlier slots
    (300, 900, 4, 2, True, True),      # window start moves inside the chunk (S > 1024)
    (700, 1500, 16, 8, True, False),   # whole chunk past the window
    (37, 0, 4, 4, False, False),       # one q head per kv head: CUDA-core kernel, ragged N
    (45, 20, 6, 2, True, True),        # three q heads per kv head: CUDA-core kernel
    (1024, 0, 2, 1, True, True),       # full prefill chunk, window edge at the last token
])
def test_batch_causal_attn_matches_oracle(ctx, oracle, N, num_prev, nq, nkv, sliding, scatter):
    rng = np.random.default_rng(N * 7 + num_prev)
    kvd = nkv * D
    S = num_prev + N
    slots = rng.permutation(4096)[:S].astype(np.uint32) if scatter else np.arange(S, dtype=np.uint32)
    kc = rng.standard_normal((4096, kvd)).astype(np.float16)
    vc = rng.standard_normal((4096, kvd)).astype(np.float16)
    q = rng.standard_normal((N, nq * D)).astype(np.float32)
    scale = 1.0 / 16.0
    ref = oracle.batch_causal_attn(q, kc.view(np.uint16), vc.view(np.uint16), slots, N, num_prev, nq, nkv, D, scale,
                                   sliding)
    lib = L.load()
    qd, kd, vd, sd, out = dev(q), dev(kc.view(np.uint16)), dev(vc.view(np.uint16)), dev(slots), empty(N * nq * D)
    call(lib.ch_batch_causal_attention, ctx.handle, qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), sd.data_ptr(), N,
         num_prev, nq, nkv, D, scale, int(sliding), out.data_ptr())
    ctx.synchronize()
    got = host(out).reshape(N, nq * D)
    assert_close(got, ref, what=f"batch causal attention N={N} prev={num_prev} {nq}/{nkv} sliding={sliding}")
    # token by token too: no row may borrow another token's window
    for t in sorted({0, N // 2, N - 1}):
        assert_close(got[t], ref[t], what=f"token {t}")


def test_batch_causal_attn_rejects_bad_shapes(ctx):
    lib = L.load()
    one = 16  # never dereferenced: the shape checks come first
    assert lib.ch_batch_causal_attention(ctx.handle, one, one, one, one, 10, 4090, 8, 1, D, 1.0, 0, one) == L.CH_EINVAL
    assert lib.ch_batch_causal_attention(ctx.handle, one, one, one, one, 10, 0, 8, 3, D, 1.0, 0, one) == L.CH_EINVAL
    assert lib.ch_batch_causal_attention(ctx.handle, one, one, one, one, 10, 0, 8, 1, 128, 1.0, 0, one) == L.CH_EINVAL
