"""GPU parity of the persistent decode-step kernel, stage by stage, against the oracle's
persistent-step order (T16 GEMV parts/slices, chunked PV).  Bit-exact everywhere:
GEMV outputs, fp32 parts, RMSNorm residuals, RoPE + KV store, SiLU*mul, argmax,
attention partials and the combined output.  All calls go through the C ABI
(spark_q4_pack_t16, spark_step_run)."""
from __future__ import annotations

import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def u16(t):
    import torch
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def t16_row(rowmap, rg, p, n, head_dim):
    if rowmap == 1:
        per = head_dim // 16
        hd, s = divmod(rg, per)
        return hd * head_dim + (8 * s + p if p < 8 else head_dim // 2 + 8 * s + p - 8)
    if rowmap == 2:
        return 8 * rg + p if p < 8 else n // 2 + 8 * rg + p - 8
    return 16 * rg + p


def np_pack_t16(qs, d, kp, rowmap=0, head_dim=0):
    """Independent numpy restatement of the T16 layout (include/spark_b200.h)."""
    n, k = qs.shape[0], qs.shape[1] * 2
    Kp, nb = k // kp, k // 32
    tiles = Kp // 64
    out = np.zeros(n * k * 9 // 16, np.uint8)
    dq = d.view(np.uint16)
    for u in range(n // 16 * kp):
        rg, kpi = divmod(u, kp)
        rows = [t16_row(rowmap, rg, p, n, head_dim) for p in range(16)]
        for t in range(tiles):
            b0 = kpi * (Kp // 32) + 2 * t
            tile = out[u * 9 * Kp + t * 576:u * 9 * Kp + (t + 1) * 576]
            for L in range(32):
                g, c = divmod(L, 4)
                ra, rb = rows[g], rows[g + 8]
                parts = [qs[ra, b0 * 16 + 4 * c:b0 * 16 + 4 * c + 4], qs[rb, b0 * 16 + 4 * c:b0 * 16 + 4 * c + 4],
                         qs[ra, b0 * 16 + 16 + 4 * c:b0 * 16 + 20 + 4 * c],
                         qs[rb, b0 * 16 + 16 + 4 * c:b0 * 16 + 20 + 4 * c]]
                tile[16 * L:16 * L + 16] = np.concatenate(parts)
                if c == 0:
                    dv = np.array([dq[ra, b0], dq[rb, b0], dq[ra, b0 + 1], dq[rb, b0 + 1]], np.uint16)
                    tile[512 + 8 * g:512 + 8 * g + 8] = dv.view(np.uint8)
    assert nb == k // 32
    return out


def _q4(n, k, seed, device="cuda"):
    import torch
    from spark_b200 import ops
    g = torch.Generator(device=device).manual_seed(seed)
    w = torch.randn((n, k), generator=g, device=device) * 0.02
    return ops.q4_quantize(w)


def _np(qs, d):
    return qs.cpu().numpy(), u16(d)


@pytest.mark.parametrize("n,k,kp,rowmap,hd", [(32, 128, 1, 0, 0), (64, 256, 2, 0, 0), (256, 128, 1, 1, 128),
                                              (64, 192, 1, 2, 0), (48, 384, 3, 0, 0)])
def test_pack_t16_matches_numpy(cuda, n, k, kp, rowmap, hd):
    from spark_b200 import step
    qs, d = _q4(n, k, seed=n + k)
    got = step.q4_pack_t16(qs, d, kp, rowmap, hd).cpu().numpy()
    want = np_pack_t16(*_np(qs, d), kp, rowmap, hd)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("n,k,kp,ks", [(64, 256, 1, 1), (48, 512, 1, 2), (160, 2560, 1, 4), (2560, 4096, 2, 4),
                                       (2560, 9728, 4, 2), (4096, 2560, 1, 1), (9728, 2560, 1, 4),
                                       # tiles per slice 1, 3, 5, 16: the odd last tile and every group batch
                                       (32, 192, 1, 3), (32, 384, 1, 2), (32, 640, 1, 2), (16, 1024, 1, 1)])
def test_t16_gemv_bitexact(cuda, oracle, n, k, kp, ks):
    import torch
    from spark_b200 import step
    qs, d = _q4(n, k, seed=7 * n + k)
    w = step.q4_pack_t16(qs, d, kp)
    x = (torch.randn(k, device="cuda") * torch.exp2(torch.randint(-6, 3, (k,), device="cuda").float())).to(
        torch.bfloat16)
    parts = step.t16_gemv(x, w, n, k, kp, ks, parts=True)
    qn, dn = _np(qs, d)
    want = oracle.t16_gemv_parts(u16(x), qn, dn, kp, ks)
    assert np.array_equal(parts.cpu().numpy().view(np.uint32), want.view(np.uint32))
    if kp == 1:
        y = step.t16_gemv(x, w, n, k, kp, ks)
        assert np.array_equal(u16(y), oracle.parts_to_bf16(want))
    # the tolerance of the reference's dequantize-then-matmul
    ref = oracle.bf16_to_f32(u16(x)).astype(np.float64) @ oracle.q4_dequantize(qn, dn).astype(np.float64).T
    got = oracle.bf16_to_f32(oracle.parts_to_bf16(want))
    assert np.all(np.abs(got - ref) <= 1e-3 + 1e-2 * np.abs(ref))


def test_step_run_rejects_bad_stages(cuda):
    """Host validation: bad slice counts, shapes and waits are refused before any launch."""
    import torch
    from spark_b200 import step
    from spark_b200._lib import SparkError
    qs, d = _q4(64, 512, seed=1)
    w = step.q4_pack_t16(qs, d, 1)
    x = torch.randn(512, device="cuda").to(torch.bfloat16)
    for kw, status in (({"ks": 5}, 2), ({"ks": 3}, 2), ({"ks": 16}, 2)):
        with pytest.raises(SparkError) as e:
            step.t16_gemv(x, w, 64, 512, 1, **kw)
        assert e.value.status == status
    prog = step.StepProgram("cuda")
    out = torch.empty(64, device="cuda", dtype=torch.bfloat16)
    prog.gemv(w, 64, 512, ks=1, a=x, out=out, wait=0)  # a stage may not wait on itself
    with pytest.raises(SparkError) as e:
        prog.finalize().launch(prog.io())
    assert e.value.status == 1


def test_t16_gemv_zero_and_tiny_blocks(cuda, oracle):
    import torch
    from spark_b200 import step
    n, k = 64, 512
    qs, d = _q4(n, k, seed=3)
    w = step.q4_pack_t16(qs, d, 1)
    x = torch.randn(k, device="cuda")
    x[:32] = 0
    x[64:96] *= 1e-35
    x = x.to(torch.bfloat16)
    y = step.t16_gemv(x, w, n, k, 1, 2)
    assert np.array_equal(u16(y), oracle.t16_gemv(u16(x), *_np(qs, d), 1, 2))


def test_t16_gemv_parts_norm_prologue(cuda, oracle):
    """x = RMSNorm(bf16(sum of fp32 parts) + b) * gamma, residual out, plain bf16 out."""
    import torch
    from spark_b200 import step
    n, k, kp_in = 256, 2560, 4
    qs, d = _q4(n, k, seed=11)
    w = step.q4_pack_t16(qs, d, 1)
    a = torch.randn((kp_in, k), device="cuda") * 0.5
    b = torch.randn(k, device="cuda").to(torch.bfloat16)
    gamma = (1 + 0.02 * torch.randn(k, device="cuda")).to(torch.bfloat16)
    res = torch.empty(k, device="cuda", dtype=torch.bfloat16)
    y = step.t16_gemv(a, w, n, k, 1, 4, a_parts=kp_in, b=b, gamma=gamma, eps=1e-6, res_out=res)
    a_bf = oracle.parts_to_bf16(a.cpu().numpy())
    want_res, xn = oracle.add_rmsnorm(a_bf, u16(b), u16(gamma), 1e-6)
    assert np.array_equal(u16(res), want_res)
    assert np.array_equal(u16(y), oracle.t16_gemv(xn, *_np(qs, d), 1, 4))


def test_t16_silu_mul_epilogue(cuda, oracle):
    import torch
    from spark_b200 import step
    i, k = 512, 2560
    qs, d = _q4(2 * i, k, seed=5)
    w = step.q4_pack_t16(qs, d, 1, step.ROWS_GATE_UP)
    x = torch.randn(k, device="cuda").to(torch.bfloat16)
    mid = torch.empty(i, device="cuda", dtype=torch.bfloat16)
    prog = step.StepProgram("cuda")
    prog.gemv(w, 2 * i, k, ks=1, a=x, epi=step.EPI_SILU_MUL, rowmap=step.ROWS_GATE_UP, out=mid)
    prog.finalize().launch(prog.io())
    gu = oracle.t16_gemv(u16(x), *_np(qs, d), 1, 1)
    assert np.array_equal(u16(mid), oracle.silu_mul(gu[:i], gu[i:]))


def test_t16_argmax_epilogue_and_finalize(cuda, oracle):
    import torch
    from spark_b200 import step
    n, k = 151936, 2560
    qs, d = _q4(n, k, seed=9)
    w = step.q4_pack_t16(qs, d, 1)
    x = torch.randn(k, device="cuda").to(torch.bfloat16)
    logits = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    key = torch.zeros(1, device="cuda", dtype=torch.int64)
    tok = torch.full((1,), -1, device="cuda", dtype=torch.int32)
    pos = torch.zeros(1, device="cuda", dtype=torch.int64)
    prog = step.StepProgram("cuda")
    prog.gemv(w, n, k, ks=1, a=x, epi=step.EPI_ARGMAX, out=logits, key=key)
    prog.finalize()
    for rep in range(2):  # the kernel leaves counters and key zero: a second launch works
        prog.launch(prog.io(key=key, token_out=tok, pos=pos))
        torch.cuda.synchronize()
        want = oracle.t16_gemv(u16(x), *_np(qs, d), 1, 1)
        assert np.array_equal(u16(logits), want)
        assert int(tok.item()) == oracle.argmax_bf16(want)
        assert int(key.item()) == 0 and int(pos.item()) == rep + 1
        c = prog.counters.cpu()
        assert int(c[:-1].abs().sum()) == 0 and int(c[-1]) == rep + 1  # stage counters zero; generation


def _rope_setup(nq=32, nkv=8, D=128, bs=128, L=300, seed=0):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    nblk = (L + bs) // bs + 2
    kc = (torch.randn((nblk, nkv, bs, D), generator=g, device="cuda")).to(torch.bfloat16)
    vc = (torch.randn((nblk, nkv, bs, D), generator=g, device="cuda")).to(torch.bfloat16)
    table = torch.randperm(nblk, generator=g, device="cuda").to(torch.int32)
    return kc, vc, table


def test_t16_rope_kvstore_epilogue(cuda, oracle):
    import torch
    from spark_b200 import step
    from spark_b200.config import SparkConfig
    from spark_b200.model import rope_cos_sin
    cfg = SparkConfig(max_position=4096)
    nq, nkv, D, h = 32, 8, 128, 2560
    n = (nq + 2 * nkv) * D
    qs, d = _q4(n, h, seed=21)
    w = step.q4_pack_t16(qs, d, 1, step.ROWS_PAIR_HALF, D)
    kc, vc, table = _rope_setup(L=1000)
    kc0, vc0 = u16(kc), u16(vc)
    cs = rope_cos_sin(cfg).cuda()
    pos_v = 777
    pos = torch.tensor([pos_v], device="cuda", dtype=torch.int64)
    q = torch.empty((nq, D), device="cuda", dtype=torch.bfloat16)
    kv_new = torch.empty((2, nkv, D), device="cuda", dtype=torch.bfloat16)
    a = torch.randn(h, device="cuda").to(torch.bfloat16)
    gamma = (1 + 0.02 * torch.randn(h, device="cuda")).to(torch.bfloat16)
    res = torch.empty(h, device="cuda", dtype=torch.bfloat16)
    prog = step.StepProgram("cuda")
    rope = {"cos_sin": cs, "pos": pos, "block_table": table, "k_cache": kc, "v_cache": vc, "q": q,
            "kv_new": kv_new, "block_size": 128, "nq": nq, "nkv": nkv}
    prog.gemv(w, n, h, ks=4, a=a, gamma=gamma, eps=1e-6, res_out=res, epi=step.EPI_ROPE_KV,
              rowmap=step.ROWS_PAIR_HALF, head_dim=D, rope=rope)
    prog.finalize().launch(prog.io())
    torch.cuda.synchronize()
    _, xn = oracle.add_rmsnorm(u16(a), None, u16(gamma), 1e-6)
    qkv = oracle.t16_gemv(xn, *_np(qs, d), 1, 4).reshape(nq + 2 * nkv, D)
    rot = oracle.rope_neox(qkv[:nq + nkv], u16(cs)[pos_v])
    assert np.array_equal(u16(q), rot[:nq])
    blk, off = int(table[pos_v // 128].item()), pos_v % 128
    kc1, vc1 = u16(kc), u16(vc)
    assert np.array_equal(kc1[blk, :, off], rot[nq:])
    assert np.array_equal(vc1[blk, :, off], qkv[nq + nkv:])
    assert np.array_equal(u16(kv_new)[0], rot[nq:]) and np.array_equal(u16(kv_new)[1], qkv[nq + nkv:])
    # nothing else in the caches changed
    kc1[blk, :, off] = kc0[blk, :, off]
    vc1[blk, :, off] = vc0[blk, :, off]
    assert np.array_equal(kc1, kc0) and np.array_equal(vc1, vc0)


# (splits x 8 kv heads > 148 CTAs: several (kv head, split) tasks per CTA)
@pytest.mark.parametrize("L,splits", [(1, 18), (17, 18), (300, 18), (2048, 18), (3000, 18), (6144, 18),
                                      (9000, 7), (129, 2), (6144, 37), (20000, 40), (32768, 25)])
def test_attention_stage_bitexact(cuda, oracle, L, splits):
    import torch
    from spark_b200 import step
    nq, nkv, D, bs = 32, 8, 128, 128
    kc, vc, table = _rope_setup(L=L, seed=L)
    pos_v = L - 1
    blk, off = int(table[pos_v // bs].item()), pos_v % bs
    kv_new = torch.stack([kc[blk, :, off], vc[blk, :, off]]).contiguous()
    g = torch.Generator(device="cuda").manual_seed(L + 1)
    q = torch.randn((nq, D), generator=g, device="cuda").to(torch.bfloat16)
    pos = torch.tensor([pos_v], device="cuda", dtype=torch.int64)
    po = torch.empty((splits, nq, D), device="cuda", dtype=torch.float32)
    pl = torch.empty((splits, nq), device="cuda", dtype=torch.float32)
    out = torch.empty((nq, D), device="cuda", dtype=torch.bfloat16)
    hc = torch.zeros(nkv, device="cuda", dtype=torch.int32)
    T = step.max_split_tokens(L, splits)
    scale = float(np.float32(1 / math.sqrt(D)))
    prog = step.StepProgram("cuda")
    prog.attention(q=q, k_cache=kc, v_cache=vc, kv_new=kv_new, block_table=table, pos=pos, splits=splits,
                   max_split_tokens=T, scale=scale, part_o=po, part_lse=pl, head_counters=hc, attn_out=out, nq=nq,
                   nkv=nkv, head_dim=D, block_size=bs)
    prog.finalize().launch(prog.io())
    torch.cuda.synchronize()
    wpo, wpl = oracle.attn_split(u16(q), u16(kc), u16(vc), table.cpu().numpy(), L, splits, scale,
                                    chunk_accs=step.CHUNK_ACCS)
    assert np.array_equal(pl.cpu().numpy().view(np.uint32), wpl.view(np.uint32))
    assert np.array_equal(po.cpu().numpy().view(np.uint32), wpo.view(np.uint32))
    assert np.array_equal(u16(out), oracle.attn_combine(wpo, wpl))
    assert bool((hc == splits).all())  # each split of every head published once
    # a second launch (next generation) gives the same result
    out.zero_()
    prog.launch(prog.io())
    torch.cuda.synchronize()
    assert np.array_equal(u16(out), oracle.attn_combine(wpo, wpl)) and bool((hc == 2 * splits).all())
