"""CPU tests that pin the oracle (oracle/spark_oracle.c) before it is trusted.

* Q4_0 quantize / dequantize against the committed gguf 0.19.0 golden vectors
  (tests/golden/q4_0_gguf.npz, made by tests/golden/make_golden.py); the Q6_K decode
  against gguf's (tests/golden/q6_k_gguf.npz).
* Slot mapping against the reference test's known-answer cases
  (tests/golden/slot_mapping_kat.npz, from tools/validation/test_slot_mapping.py).
* The canonical-order GEMV, attention, combine, norm, RoPE and SiLU against
  independent float64 numpy restatements, within the tolerances the north star
  states (GEMV rel 1e-2 / abs 1e-3, attention abs 2e-2).
"""
from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"


def bf16(a):
    import oracle as O
    return O.f32_to_bf16(a)


def f32(b):
    import oracle as O
    return O.bf16_to_f32(b)


# ----------------------------------------------------------------------------- Q4_0 golden vectors
def test_q4_quantize_matches_gguf_golden(oracle):
    z = np.load(GOLDEN / "q4_0_gguf.npz")
    names = sorted({k.split(".")[0] for k in z.files})
    assert {"normal", "wide", "zeros", "ties", "large"} <= set(names)
    for n in names:
        w, blocks = z[n + ".w"], z[n + ".blocks"]
        qs, d = oracle.q4_quantize(w)
        assert np.array_equal(oracle.q4_join(qs, d).reshape(-1), blocks.reshape(-1)), n


def test_q4_dequantize_matches_gguf_golden(oracle):
    z = np.load(GOLDEN / "q4_0_gguf.npz")
    for n in sorted({k.split(".")[0] for k in z.files}):
        w, blocks, deq = z[n + ".w"], z[n + ".blocks"], z[n + ".deq"]
        qs, d = oracle.q4_split(blocks, w.shape[0], w.shape[1])
        got = oracle.q4_dequantize(qs, d)
        assert np.array_equal(got.view(np.uint32), deq.reshape(got.shape).view(np.uint32)), n


# ----------------------------------------------------------------------------- Q6_K golden vectors
def test_q6k_dequantize_matches_gguf_golden(oracle):
    """gguf 0.19.0 decode of random / edge-case Q6_K super-blocks, bit for bit."""
    z = np.load(GOLDEN / "q6_k_gguf.npz")
    names = sorted({k.split(".")[0] for k in z.files})
    assert {"normal", "edges", "rows"} <= set(names)
    for n in names:
        got = oracle.q6k_dequantize(z[n + ".blocks"])
        want = z[n + ".deq"].reshape(-1)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), n


def test_q6k_gemv_order_within_tolerance(oracle):
    """The Q6_K GEMV order against a float64 dequantize-then-matmul of gguf's decode."""
    z = np.load(GOLDEN / "q6_k_gguf.npz")
    blocks = z["rows.blocks"].reshape(4, 10 * 210)  # 4 rows of K = 2560
    rng = np.random.default_rng(0)
    for amp in (1e-3, 1.0, 1e3):
        x = bf16((rng.standard_normal(2560) * amp).astype(np.float32))
        for kp, ks in ((1, 1), (1, 2), (2, 5)):
            y = f32(oracle.parts_to_bf16(oracle.q6k_gemv_parts(x, blocks, 4, 2560, kp, ks)))
            ref = oracle.q6k_dequantize(blocks).reshape(4, 2560).astype(np.float64) @ f32(x).astype(np.float64)
            assert np.all(np.abs(y - ref) <= 1e-3 * amp + 1e-2 * np.abs(ref)), (amp, kp, ks)


def test_q4_split_join_roundtrip(oracle):
    z = np.load(GOLDEN / "q4_0_gguf.npz")
    blocks = z["normal.blocks"]
    qs, d = oracle.q4_split(blocks, 64, 512)
    assert np.array_equal(oracle.q4_join(qs, d), blocks.reshape(64, -1))
    # unpack_q4 semantics (integration/weights.py:34-40): low nibbles first, then high
    q = np.concatenate((qs.reshape(64, 16, 16) & 15, qs.reshape(64, 16, 16) >> 4), axis=-1).reshape(64, 512)
    deq = oracle.q4_dequantize(qs, d)
    scale = np.repeat(oracle.bf16_to_f32(np.zeros(1, np.uint16)), 1)  # noqa: F841 (shape check only)
    dd = d.view(np.float16).astype(np.float32).repeat(32, axis=1)
    assert np.array_equal(deq, dd * (q.astype(np.float32) - 8))


# ----------------------------------------------------------------------------- slot mapping KAT
def test_slot_mapping_kat(oracle):
    z = np.load(GOLDEN / "slot_mapping_kat.npz")
    maximum = int(z["maximum"])
    for ci, (count, offset) in enumerate(z["cases"]):
        pos = np.arange(count, dtype=np.int64) + offset
        for gi, size in enumerate(z["sizes"]):
            got = oracle.slot_mapping(pos, z["tables"][gi], int(size), maximum)
            exp = z[f"case{ci}.group{gi}"]
            assert np.array_equal(got[:count], exp), (ci, gi)
            assert np.all(got[count:] == -1)


def test_slot_mapping_query_window(oracle):
    table = np.arange(8, dtype=np.int32)[::-1].copy()
    pos = np.arange(10, dtype=np.int64) + 120
    out = oracle.slot_mapping(pos, table, 128, 16, start=2, end=7)
    assert np.all(out[:2] == -1) and np.all(out[7:] == -1)
    assert out[2] == table[122 // 128] * 128 + 122 % 128
    assert out[6] == table[126 // 128] * 128 + 126


# ----------------------------------------------------------------------------- exp / log
def test_exp_log_accuracy(oracle):
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.uniform(-87, 88, 4000), rng.uniform(-1, 1, 1000), [0.0, -0.0, 1e-30, -50.0]])
    for x in xs.astype(np.float32):
        got = oracle.exp(float(x))
        ref = math.exp(float(x))
        assert abs(got - ref) <= 2 * np.spacing(np.float32(ref)), x
    for x in np.exp(rng.uniform(-80, 80, 3000)).astype(np.float32):
        got, ref = oracle.log(float(x)), math.log(float(x))
        assert abs(got - ref) <= 2 * np.spacing(np.float32(abs(ref)) if ref != 0 else np.float32(1e-7)), x
    assert oracle.exp(-200.0) == 0.0 and math.isinf(oracle.exp(100.0))
    assert oracle.log(1.0) == 0.0 and math.isinf(oracle.log(0.0))


# ----------------------------------------------------------------------------- GEMV
def _q4_setup(n, k, seed=0, batch=1):
    import oracle as O
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    x = bf16(rng.standard_normal((batch, k)).astype(np.float32))
    qs, d = O.q4_quantize(w)
    return x, qs, d


@pytest.mark.parametrize("n,k,batch", [(64, 256, 1), (96, 2560, 1), (32, 9728, 1), (48, 544, 3)])
def test_gemv_oracle_vs_dequant_matmul(oracle, n, k, batch):
    """The reference's PyTorch path: gguf dequantize -> matmul (integration/weights.py:28-31)."""
    x, qs, d = _q4_setup(n, k, batch=batch)
    y = f32(oracle.q4_gemv(x, qs, d))
    w = oracle.q4_dequantize(qs, d).astype(np.float64)
    ref = f32(x).astype(np.float64) @ w.T
    assert np.all(np.abs(y - ref) <= 1e-3 + 1e-2 * np.abs(ref))
    # rounding only at the bf16 output: the unrounded sums agree to ~fp32 accuracy
    yf = oracle.q4_gemv_f32(f32(x), qs, d)
    assert np.max(np.abs(yf - ref)) < 1e-4 * max(1.0, np.abs(ref).max())


def _stage_np(xf, s0=14):
    """Independent numpy restatement of the documented activation staging."""
    X = np.zeros(xf.size, np.int64)
    sx = np.ones(xf.size // 32, np.float32)
    C = np.zeros(xf.size // 32, np.int64)
    for b in range(xf.size // 32):
        blk = xf[32 * b:32 * b + 32].astype(np.float32)
        M = np.abs(blk).max()
        if not (M >= np.float32(2.0 ** -100)) or not np.isfinite(M):
            continue
        e = int(np.floor(np.log2(np.float64(M))))
        S = s0 - e
        X[32 * b:32 * b + 32] = np.rint(blk.astype(np.float64) * 2.0 ** S).astype(np.int64)
        sx[b] = np.float32(2.0 ** -S)
        C[b] = 8 * X[32 * b:32 * b + 32].sum()
    return X, sx, C


def test_stage_x_is_exact_fixed_point(oracle):
    rng = np.random.default_rng(9)
    x = f32(bf16(rng.standard_normal(2560).astype(np.float32) * np.exp2(rng.integers(-12, 4, 2560))))
    X, sx, C = oracle.q4_stage_x(x)
    eX, esx, eC = _stage_np(x)
    assert np.array_equal(X.astype(np.int64), eX) and np.array_equal(sx, esx) and np.array_equal(C, eC)
    assert np.abs(X).max() <= 32640
    # elements within 2^7 of their block maximum are represented exactly
    xb, Xb = x.reshape(-1, 32), X.reshape(-1, 32).astype(np.float64) * sx[:, None]
    big = np.abs(xb) >= np.abs(xb).max(axis=1, keepdims=True) / 128
    assert np.array_equal(Xb[big], xb[big].astype(np.float64))
    # all-zero and tiny blocks stage to zero
    X0, sx0, C0 = oracle.q4_stage_x(np.zeros(64, np.float32))
    assert not X0.any() and np.all(sx0 == 1.0) and not C0.any()


def test_gemv_canonical_order_is_documented(oracle):
    """Re-derive rows in Python from the documented order and compare bits."""
    x, qs, d = _q4_setup(3, 1024, seed=3)
    xf = f32(x)[0]
    X, sx, C = _stage_np(xf)
    nb = 1024 // 32
    dd = d.view(np.float16).astype(np.float32)
    rows = []
    for r in range(3):
        lanes = []
        for lane in range(16):
            acc = np.float32(0)
            for b in range(lane, nb, 16):
                q = qs[r, b * 16:(b + 1) * 16].astype(np.int64)
                P = int(((q & 15) * X[32 * b:32 * b + 16]).sum() + ((q >> 4) * X[32 * b + 16:32 * b + 32]).sum() - C[b])
                assert abs(P) < 2 ** 24
                ds = np.float32(dd[r, b] * sx[b])
                # fma(ds, P, acc): ds * P is exact in float64 (11+24 significant bits < 53)
                acc = np.float32(np.float64(ds) * np.float64(P) + np.float64(acc))
            lanes.append(acc)
        v = np.array(lanes, np.float32)
        for off in (8, 4, 2, 1):
            v = (v + v[np.arange(16) ^ off]).astype(np.float32)
        rows.append(v[0])
    got = oracle.q4_gemv_f32(xf, qs, d)[0]
    assert np.array_equal(np.array(rows, np.float32).view(np.uint32), got.view(np.uint32))


@pytest.mark.parametrize("kp,ks", [(1, 1), (1, 4), (2, 2), (4, 1)])
def test_t16_gemv_order_is_documented(oracle, kp, ks):
    """Persistent-step order: S = 13 - e staging, KP parts of KS slices, each slice four
    block chains (blocks b0 + c, b0 + c + 4, ...) summed as (c0 + c1) + (c2 + c3)."""
    x, qs, d = _q4_setup(3, 1024, seed=5)
    xf = f32(x)[0]
    X, sx, C = _stage_np(xf, s0=13)
    assert np.abs(X).max() <= 16320
    # X splits into two signed bytes: X = 256 h + l, h, l in [-128, 127]
    lo = ((X + 128) & 255) - 128
    hi = (X - lo) // 256
    assert np.abs(hi).max() <= 64 and np.array_equal(256 * hi + lo, X)
    nb = 1024 // 32
    bpp, bps = nb // kp, nb // kp // ks
    dd = d.view(np.float16).astype(np.float32)
    want = np.zeros((kp, 3), np.float32)
    for r in range(3):
        for p in range(kp):
            part = np.float32(0)
            for sl in range(ks):
                chains = [np.float32(0)] * 4
                b0 = p * bpp + sl * bps
                for b in range(b0, b0 + bps):
                    q = qs[r, b * 16:(b + 1) * 16].astype(np.int64)
                    P = int(((q & 15) * X[32 * b:32 * b + 16]).sum() + ((q >> 4) * X[32 * b + 16:32 * b + 32]).sum()
                            - C[b])
                    ds = np.float32(dd[r, b] * sx[b])
                    c = (b - b0) & 3
                    chains[c] = np.float32(np.float64(ds) * np.float64(P) + np.float64(chains[c]))
                acc = np.float32(np.float32(chains[0] + chains[1]) + np.float32(chains[2] + chains[3]))
                part = acc if sl == 0 else np.float32(part + acc)
            want[p, r] = part
    got = oracle.t16_gemv_parts(x[0], qs, d, kp, ks)
    assert np.array_equal(want.view(np.uint32), got.view(np.uint32))
    y = oracle.t16_gemv(x[0], qs, d, kp, ks)
    tot = want[0].copy()
    for p in range(1, kp):
        tot = (tot + want[p]).astype(np.float32)
    assert np.array_equal(y, bf16(tot))


@pytest.mark.parametrize("n,k,kp,ks", [(64, 2560, 1, 4), (48, 4096, 2, 4), (32, 9728, 4, 2)])
def test_t16_gemv_vs_dequant_matmul(oracle, n, k, kp, ks):
    """The persistent-step order meets the GEMV tolerance (rel 1e-2 / abs 1e-3) against the
    reference's dequantize-then-matmul."""
    x, qs, d = _q4_setup(n, k, seed=n + k)
    w = oracle.q4_dequantize(qs, d)
    ref = f32(x)[0].astype(np.float64) @ w.astype(np.float64).T
    y = f32(oracle.t16_gemv(x[0], qs, d, kp, ks))
    assert np.all(np.abs(y - ref) <= 1e-3 + 1e-2 * np.abs(ref))


# ----------------------------------------------------------------------------- norm / rope / silu
def test_add_rmsnorm_vs_float64(oracle):
    rng = np.random.default_rng(1)
    a, b = bf16(rng.standard_normal(2560)), bf16(rng.standard_normal(2560))
    g = bf16(1 + 0.02 * rng.standard_normal(2560))
    res, y = oracle.add_rmsnorm(a, b, g, 1e-6)
    s = f32(a).astype(np.float64) + f32(b)
    assert np.array_equal(res, bf16(s.astype(np.float32)))
    ref = s / np.sqrt(np.mean(s * s) + 1e-6) * f32(g)
    assert np.max(np.abs(f32(y) - ref)) <= 1e-2 * np.abs(ref).max()
    _, y0 = oracle.add_rmsnorm(a, None, g, 1e-6)
    s0 = f32(a).astype(np.float64)
    assert np.allclose(f32(y0), s0 / np.sqrt(np.mean(s0 * s0) + 1e-6) * f32(g), rtol=1e-2, atol=1e-2)


def test_rope_neox(oracle):
    rng = np.random.default_rng(2)
    x = bf16(rng.standard_normal((4, 128)))
    pos = 777
    inv = 1.0 / (1e6 ** (np.arange(0, 128, 2) / 128))
    ang = pos * inv
    cs = bf16(np.concatenate([np.cos(ang), np.sin(ang)]).astype(np.float32))
    out = f32(oracle.rope_neox(x, cs))
    xf, c, s = f32(x), f32(cs)[:64], f32(cs)[64:]
    ref = np.concatenate([xf[:, :64] * c - xf[:, 64:] * s, xf[:, 64:] * c + xf[:, :64] * s], axis=1)
    assert np.max(np.abs(out - ref)) < 2e-2


def test_silu_mul(oracle):
    rng = np.random.default_rng(3)
    g, u = bf16(rng.standard_normal(4096) * 3), bf16(rng.standard_normal(4096))
    out = f32(oracle.silu_mul(g, u))
    gf = f32(g).astype(np.float64)
    ref = gf / (1 + np.exp(-gf)) * f32(u)
    assert np.max(np.abs(out - ref)) < 2e-2 * max(1, np.abs(ref).max())


# ----------------------------------------------------------------------------- attention
def _paged(rng, L, nkv=8, D=128, bs=128, pool_factor=4):
    nblk = (L + bs - 1) // bs
    pool = max(1, nblk * pool_factor)
    kc = bf16(rng.standard_normal((pool, nkv, bs, D)).astype(np.float32))
    vc = bf16(rng.standard_normal((pool, nkv, bs, D)).astype(np.float32))
    table = rng.permutation(pool)[:max(nblk, 1)].astype(np.int32)
    return kc, vc, table


def _attn_ref64(q, kc, vc, table, L, scale):
    nq, D = q.shape
    nkv, bs = kc.shape[1], kc.shape[2]
    G = nq // nkv
    t = np.arange(L)
    blk, off = table[t // bs], t % bs
    out = np.zeros((nq, D))
    for h in range(nq):
        hk = h // G
        K = f32(kc[blk, hk, off]).astype(np.float64)
        V = f32(vc[blk, hk, off]).astype(np.float64)
        s = K @ f32(q[h]).astype(np.float64) * scale
        p = np.exp(s - s.max())
        out[h] = p @ V / p.sum()
    return out


@pytest.mark.parametrize("L,splits", [(1, 16), (100, 16), (2048, 16), (600, 7), (300, 64)])
def test_attention_split_combine_vs_float64(oracle, L, splits):
    rng = np.random.default_rng(L)
    kc, vc, table = _paged(rng, L)
    q = bf16(rng.standard_normal((32, 128)).astype(np.float32))
    scale = float(np.float32(1 / math.sqrt(128)))
    po, pl = oracle.attn_split(q, kc, vc, table, L, splits, scale)
    out = f32(oracle.attn_combine(po, pl))
    ref = _attn_ref64(q, kc, vc, table, L, scale)
    assert np.max(np.abs(out - ref)) < 2e-2
    T = oracle.split_tokens(L, splits)
    empty = [s for s in range(splits) if s * T >= L]
    assert all(np.all(np.isneginf(pl[s])) and np.all(po[s] == 0) for s in empty)


@pytest.mark.parametrize("L,splits,W", [(3000, 18, 11), (700, 18, 11), (64, 74, 11), (2049, 5, 3), (2049, 2, 11)])
def test_attention_warp_ranges_vs_float64(oracle, L, splits, W):
    """Persistent-step order (each split cut into W token ranges with their own softmax,
    merged by their maxima) meets abs 2e-2 and agrees with the one-range order to within
    the bf16 rounding of P (each range rounds p relative to its own maximum)."""
    rng = np.random.default_rng(L + W)
    kc, vc, table = _paged(rng, L)
    q = bf16(rng.standard_normal((32, 128)).astype(np.float32))
    scale = float(np.float32(1 / math.sqrt(128)))
    po, pl = oracle.attn_split(q, kc, vc, table, L, splits, scale, chunk_accs=W)
    out = f32(oracle.attn_combine(po, pl))
    assert np.max(np.abs(out - _attn_ref64(q, kc, vc, table, L, scale))) <= 2e-2
    po0, pl0 = oracle.attn_split(q, kc, vc, table, L, splits, scale)
    assert np.array_equal(np.isneginf(pl), np.isneginf(pl0))
    fin = np.isfinite(pl0)
    assert np.allclose(pl[fin], pl0[fin], rtol=0, atol=1e-5)
    assert np.allclose(po, po0, rtol=1e-2, atol=4e-3)


def test_attention_warp_ranges_order_is_documented(oracle):
    """numpy restatement of the persistent-step order, compared bit for bit: ranges of
    C = roundup(ceil(n / W), 512 / D) tokens, per-range max / exp / 32-lane sum / bf16 P /
    ascending P V, then the merge in range order."""
    rng = np.random.default_rng(17)
    L, splits, W, D = 300, 2, 11, 128
    kc, vc, table = _paged(rng, L)
    q = bf16(rng.standard_normal((32, D)).astype(np.float32))
    scale = float(np.float32(1 / math.sqrt(D)))
    po, pl = oracle.attn_split(q, kc, vc, table, L, splits, scale, chunk_accs=W)
    T = oracle.split_tokens(L, splits)
    bs = kc.shape[2]
    lanes = D // 16
    ninf = np.float32(-np.inf)
    for s in range(splits):
        t0, t1 = s * T, min((s + 1) * T, L)
        n = t1 - t0
        C = -(-(-(-n // W)) // (512 // D)) * (512 // D)
        for hq in (0, 5, 31):
            hk = hq // 4
            qf = f32(q[hq])
            ms, ls, os = [], [], []
            for w in range(W):
                a, b = w * C, min(w * C + C, n)
                if a >= n:
                    ms.append(ninf), ls.append(np.float32(0)), os.append(np.zeros(D, np.float32))
                    continue
                sc = []
                for i in range(a, b):
                    t = t0 + i
                    k = f32(kc[table[t // bs], hk, t % bs])
                    per = D // 2 // lanes
                    lane = []
                    for j in range(lanes):
                        a0 = a1 = np.float32(0)
                        for part in range(2):
                            base = part * D // 2 + per * j
                            for m in range(0, per, 2):
                                a0 = np.float32(np.float64(qf[base + m]) * np.float64(k[base + m]) + np.float64(a0))
                                a1 = np.float32(np.float64(qf[base + m + 1]) * np.float64(k[base + m + 1])
                                                + np.float64(a1))
                        lane.append(np.float32(a0 + a1))
                    v = np.array(lane, np.float32)
                    off = lanes // 2
                    while off:
                        v = (v + v[np.arange(lanes) ^ off]).astype(np.float32)
                        off //= 2
                    sc.append(np.float32(v[0] * np.float32(scale)))
                m = max(sc)
                lane = np.zeros(32, np.float32)
                P = []
                for i, x in enumerate(sc):
                    pv = np.float32(oracle.exp(float(np.float32(x - m))))
                    lane[i % 32] = np.float32(lane[i % 32] + pv)
                    P.append(f32(bf16(np.array([pv], np.float32)))[0])
                off = 16
                while off:
                    lane = (lane + lane[np.arange(32) ^ off]).astype(np.float32)
                    off //= 2
                o = np.zeros(D, np.float32)
                for i in range(a, b):
                    t = t0 + i
                    v = f32(vc[table[t // bs], hk, t % bs])
                    o = (np.float64(P[i - a]) * v.astype(np.float64) + o.astype(np.float64)).astype(np.float32)
                ms.append(np.float32(m)), ls.append(lane[0]), os.append(o)
            M = max(ms)
            Lsum = np.float32(0)
            O = np.zeros(D, np.float32)
            for w in range(W):
                f = np.float32(0) if ms[w] == ninf else np.float32(oracle.exp(float(np.float32(ms[w] - M))))
                Lsum = np.float32(Lsum + np.float32(f * ls[w]))
                O = (O + (f * os[w]).astype(np.float32)).astype(np.float32)
            want_o = (O / Lsum).astype(np.float32)
            want_l = np.float32(np.float32(oracle.log(float(Lsum))) + M)
            assert np.array_equal(po[s, hq].view(np.uint32), want_o.view(np.uint32)), (s, hq)
            assert np.float32(pl[s, hq]).view(np.uint32) == want_l.view(np.uint32), (s, hq)


def test_combine_single_split_identity(oracle):
    rng = np.random.default_rng(5)
    po = rng.standard_normal((1, 4, 128)).astype(np.float32)
    pl = rng.standard_normal((1, 4)).astype(np.float32)
    assert np.array_equal(oracle.attn_combine(po, pl), bf16(po[0]))


def test_argmax_ties_lowest_index(oracle):
    lg = bf16(np.array([0.5, 2.0, -1.0, 2.0, 1.0], np.float32))
    assert oracle.argmax_bf16(lg) == 1
