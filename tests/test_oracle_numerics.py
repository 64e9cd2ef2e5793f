"""Oracle self-checks on CPU: number formats against numpy, Q4/Q8 block decode
against an independent numpy float64 evaluation, quantizer round trips, and
seeded-generator determinism."""
import numpy as np
import pytest


def test_f16_conversion_matches_numpy(oracle):
    l = oracle.lib()
    rng = np.random.default_rng(0)
    vals = np.concatenate([rng.standard_normal(2000) * s for s in (1e-6, 1e-3, 1, 100, 6e4)]).astype(np.float32)
    vals = np.concatenate([vals, np.float32([0.0, -0.0, 65504, 65519.99, 65520, 1e-8, 2**-24, 2**-25, 3 * 2**-26])])
    for v in vals:
        h = l.or_f16_from_f32(float(v))
        assert h == int(np.float16(v).view(np.uint16)), v
        assert l.or_f16_to_f32(h) == float(np.float16(v))


def decode_q4(W, M, K):
    nb = K // 32
    Wb = W.reshape(M, nb, 5)
    d = (Wb[:, :, 0] & 0xFFFF).astype(np.uint16).view(np.float16).astype(np.float64)
    nib = np.stack([(Wb[:, :, 1 + w] >> (4 * k)) & 0xF for w in range(4) for k in range(8)], axis=-1)
    return (nib.astype(np.float64) - 8.0) * d[:, :, None]  # [M, nb, 32]


def test_gemv_q4_matches_float64(oracle):
    M, K = 64, 256
    W = oracle.gen_q4(M, K, oracle.tensor_seed(7, 0, 0))
    x = oracle.gen_f32(K, 99)
    y = oracle.gemv_q4(W, x, M, K)
    ref = decode_q4(W, M, K).reshape(M, K) @ x.astype(np.float64)
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 1e-6


def test_gemv_q8_matches_float64(oracle):
    M, K = 48, 128
    emb = oracle.gen_bf16(M * K, 5, 0.0, 0.02)
    W = oracle.quantize_matrix(emb, M, K, 8)
    Wb = W.reshape(M, K // 32, 9)
    s = Wb[:, :, 0].copy().view(np.float32).astype(np.float64)
    q = Wb[:, :, 1:].copy().view(np.int8).reshape(M, K // 32, 32).astype(np.float64)
    x = oracle.gen_f32(K, 3)
    ref = (q * s[:, :, None]).reshape(M, K) @ x.astype(np.float64)
    y = oracle.gemv_q8(W, x, M, K)
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 1e-6
    # and the dequantized rows approximate the bf16 source
    src = oracle.bf16_to_f32(emb).reshape(M, K)
    assert np.abs((q * s[:, :, None]).reshape(M, K) - src).max() <= np.abs(src).max() / 127 * 0.51 + 1e-9


def test_quantize_q4_roundtrip(oracle):
    M, K = 16, 128
    src = oracle.gen_bf16(M * K, 11, 0.0, 0.05)
    W = oracle.quantize_matrix(src, M, K, 4)
    f = oracle.bf16_to_f32(src).reshape(M, K // 32, 32).astype(np.float64)
    deq = decode_q4(W, M, K)
    amax = np.abs(f).max(axis=2, keepdims=True)
    # step d = amax/8 (f16): error <= d/2 except the clamp at +amax (q=16 -> 15): <= d
    assert np.all(np.abs(deq - f) <= amax / 8 * 1.01 + 1e-12)
    # the stored min is -8d
    Wb = W.reshape(M, K // 32, 5)
    d = (Wb[:, :, 0] & 0xFFFF).astype(np.uint16).view(np.float16).astype(np.float32)
    mn = (Wb[:, :, 0] >> 16).astype(np.uint16).view(np.float16).astype(np.float32)
    assert np.allclose(mn, -8 * d, rtol=2e-3)


def test_generator_is_deterministic(oracle):
    a = oracle.gen_q4(32, 64, 1234)
    b = oracle.gen_q4(32, 64, 1234)
    c = oracle.gen_q4(32, 64, 1235)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    z = np.array([oracle.lib().or_gen_normal(5, 1, i) for i in range(20000)])
    assert abs(z.mean()) < 0.03 and abs(z.std() - 1.0) < 0.03
    nib = np.stack([(a[:, 1:5] >> (4 * k)) & 0xF for k in range(8)]).ravel()
    assert nib.min() == 0 and nib.max() == 15


def test_topk_tie_break_and_softcap(oracle):
    lg = np.zeros(1000, np.float32)
    lg[[5, 7, 900]] = 3.0
    lg[42] = 4.0
    ids, vals = oracle.topk64(lg)
    assert list(ids[:4]) == [42, 5, 7, 900]
    assert np.isclose(vals[0], 30 * np.tanh(4.0 / 30), rtol=1e-6)
    assert list(ids[4:8]) == [0, 1, 2, 3]  # ties at 0.0 by lowest index
    assert oracle.lib().or_argmax(oracle.p(lg, oracle.f32), lg.size) == 42


def test_attention_softmax_properties(oracle):
    nq, nkv, D = 4, 2, 256
    rng = np.random.default_rng(1)
    kc = rng.standard_normal((4096, nkv * D)).astype(np.float16).view(np.uint16)
    vc = np.ones((4096, nkv * D), np.float16).view(np.uint16)
    q = rng.standard_normal(nq * D).astype(np.float32)
    out = oracle.decode_attn(q, kc, vc, np.arange(100, 140), nq, nkv, D, 1 / 16)
    assert np.allclose(out, 1.0, atol=1e-5)  # convex combination of all-ones V
    out0 = oracle.decode_attn(q, kc, vc, np.array([], np.uint32), nq, nkv, D, 1 / 16)
    assert np.all(out0 == 0)  # empty list: 0 * 1/(0 + 1e-9) (decode_attn.wgsl:117)
