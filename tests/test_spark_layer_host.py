"""Host-side pins of the Spark layer features: the GELU table (the reference's recipe,
integration/model.py:12-16) equals the oracle's and lies within one bf16 step of the
float64 exact-erf GELU above x = -4 (below, 1 + erf cancels in fp32 in the reference's
own table too); the bf16 sigmoid gate matches float64 within one bf16 step; the
oracle's sliding-window attention matches a direct float64 softmax over the window and
ignores every position before it."""
from __future__ import annotations

import math

import numpy as np


def _bf16_to_f64(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def test_gelu_table_product_equals_oracle_and_exact(oracle):
    import torch
    from spark_b200 import step
    t = step.gelu_table("cpu").view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(t, oracle.gelu_table())
    inputs = np.concatenate([np.arange(0x3B00, 0x4300), np.arange(0xBB00, 0xC300)]).astype(np.uint16)
    x = _bf16_to_f64(inputs)
    exact = np.array([0.5 * v * math.erfc(-v / math.sqrt(2.0)) for v in x])
    got = _bf16_to_f64(t)
    ulp = np.abs(exact) * 2.0 ** -7
    live = x > -4.0
    assert np.all(np.abs(got[live] - exact[live]) <= ulp[live] + 1e-45)
    assert np.all(np.abs(got[~live] - exact[~live]) <= np.abs(x[~live]) * 2.0 ** -23)


def test_sigmoid_gate_close_to_exact(oracle):
    bits = np.arange(0, 65536, 97, dtype=np.uint32).astype(np.uint16)
    x = _bf16_to_f64(bits)
    ok = np.isfinite(x)
    got = _bf16_to_f64(oracle.sigmoid_bf16(bits[ok]))
    exact = 1.0 / (1.0 + np.exp(-np.clip(x[ok], -700, 700)))
    assert np.all(np.abs(got - exact) <= np.maximum(exact, 1e-38) * 2.0 ** -8)


def test_window_attention_ignores_positions_before_window(oracle):
    rng = np.random.default_rng(3)
    nq, nkv, D, bs, L = 8, 2, 256, 128, 700
    nblk = L // bs + 2

    def f(*s):
        return rng.standard_normal(s).astype(np.float32)

    kc = oracle.f32_to_bf16(f(nblk, nkv, bs, D))
    vc = oracle.f32_to_bf16(f(nblk, nkv, bs, D))
    q = oracle.f32_to_bf16(f(nq, D))
    table = rng.permutation(nblk).astype(np.int32)
    scale = float(np.float32(1 / 16))
    po, pl = oracle.attn_split(q, kc, vc, table, L, 5, scale, chunk_accs=11, window=513)
    out = oracle.bf16_to_f32(oracle.attn_combine(po, pl)).astype(np.float64)
    pos = np.arange(L - 513, L)
    K = oracle.bf16_to_f32(kc[table[pos // bs], :, pos % bs]).astype(np.float64)
    V = oracle.bf16_to_f32(vc[table[pos // bs], :, pos % bs]).astype(np.float64)
    Q = oracle.bf16_to_f32(q).astype(np.float64)
    for h in range(nq):
        s = K[:, h // (nq // nkv)] @ Q[h] * scale
        p = np.exp(s - s.max())
        want = (p / p.sum()) @ V[:, h // (nq // nkv)]
        assert np.max(np.abs(out[h] - want)) < 2e-2
    kc2 = kc.copy()
    kc2[table[(L - 600) // bs], :, (L - 600) % bs] ^= 0x1234
    po2, pl2 = oracle.attn_split(q, kc2, vc, table, L, 5, scale, chunk_accs=11, window=513)
    assert np.array_equal(po, po2) and np.array_equal(pl, pl2)
