"""GPU parity of the Spark layer features in the persistent step (the reference's Spark
architecture, plugin/spark2_5.py:140-241): head_dim 256 / 16 q : 4 kv heads, partial
RoPE (rotary 64 of 256 on full-attention layers), sliding-window attention, the
headwise sigmoid output gate, and exact-erf GELU * mul.  Bit-exact against the oracle
(oracle.rope_partial, sigmoid_bf16, attn_split(window=...), attn_combine(gate=...),
gelu_mul); all launches through the C ABI (spark_q4_pack_t16, spark_step_run)."""
from __future__ import annotations

import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

NQ, NKV, D, BS = 16, 4, 256, 128


def u16(t):
    import torch
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def t16_row_x(rg, p, n, head_dim, rot):
    """Spark qkv rows of position p of row group rg (include/spark_b200.h, ROWS_PAIR_HALF)."""
    r = rot or head_dim
    per = head_dim // 16
    hd, s = divmod(rg, per)
    if (hd + 1) * head_dim > n:  # gate rows after the last whole head
        return hd * head_dim + 16 * s + p
    if s < r // 16:
        return hd * head_dim + (8 * s + p if p < 8 else r // 2 + 8 * s + p - 8)
    return hd * head_dim + r + 16 * (s - r // 16) + p


def np_pack_qkv(qs, d, head_dim, rot):
    """numpy restatement of the T16 layout for the Spark qkv rowmap (kp 1)."""
    n, k = qs.shape[0], qs.shape[1] * 2
    tiles = k // 64
    out = np.zeros(n * k * 9 // 16, np.uint8)
    dq = d.view(np.uint16)
    for u in range(n // 16):
        rows = [t16_row_x(u, p, n, head_dim, rot) for p in range(16)]
        for t in range(tiles):
            b0 = 2 * t
            tile = out[u * 9 * k + t * 576:u * 9 * k + (t + 1) * 576]
            for L in range(32):
                g, c = divmod(L, 4)
                ra, rb = rows[g], rows[g + 8]
                tile[16 * L:16 * L + 16] = np.concatenate([
                    qs[ra, b0 * 16 + 4 * c:b0 * 16 + 4 * c + 4], qs[rb, b0 * 16 + 4 * c:b0 * 16 + 4 * c + 4],
                    qs[ra, b0 * 16 + 16 + 4 * c:b0 * 16 + 20 + 4 * c], qs[rb, b0 * 16 + 16 + 4 * c:b0 * 16 + 20 + 4 * c]])
                if c == 0:
                    dv = np.array([dq[ra, b0], dq[rb, b0], dq[ra, b0 + 1], dq[rb, b0 + 1]], np.uint16)
                    tile[512 + 8 * g:512 + 8 * g + 8] = dv.view(np.uint8)
    return out


def _q4(n, k, seed, scale=0.02):
    import torch
    from spark_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(seed)
    return ops.q4_quantize(torch.randn((n, k), generator=g, device="cuda") * scale)


def _np(qs, d):
    return qs.cpu().numpy(), u16(d)


def _caches(L, seed, nblk_extra=2):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    nblk = (L + BS) // BS + nblk_extra
    kc = torch.randn((nblk, NKV, BS, D), generator=g, device="cuda").to(torch.bfloat16)
    vc = torch.randn((nblk, NKV, BS, D), generator=g, device="cuda").to(torch.bfloat16)
    table = torch.randperm(nblk, generator=g, device="cuda").to(torch.int32)
    return kc, vc, table


@pytest.mark.parametrize("rot", [0, 64])
def test_pack_t16_spark_qkv_matches_numpy(cuda, rot):
    from spark_b200 import step
    n = (NQ + 2 * NKV) * D + 16  # heads, then the 16 gate rows
    qs, d = _q4(n, 128, seed=3 + rot)
    got = step.q4_pack_t16(qs, d, 1, step.ROWS_PAIR_HALF, D, rot).cpu().numpy()
    assert np.array_equal(got, np_pack_qkv(*_np(qs, d), D, rot))


def test_gelu_mul_epilogue(cuda, oracle):
    """Gate values over every region of the GELU table (|x| < 2^-9, the table, |x| >= 128)."""
    import torch
    from spark_b200 import ops, step
    i, k = 1024, 2560
    g = torch.Generator(device="cuda").manual_seed(12)
    # row scales 2^-16 .. 2^8 so the gate values reach every range of the table
    rs = torch.exp2(torch.randint(-16, 9, (2 * i, 1), generator=g, device="cuda").float()) * 0.02
    qs, d = ops.q4_quantize(torch.randn((2 * i, k), generator=g, device="cuda") * rs)
    w = step.q4_pack_t16(qs, d, 1, step.ROWS_GATE_UP)
    x = torch.randn(k, generator=g, device="cuda").to(torch.bfloat16)
    table = step.gelu_table("cuda")
    mid = torch.empty(i, device="cuda", dtype=torch.bfloat16)
    prog = step.StepProgram("cuda")
    prog.gemv(w, 2 * i, k, ks=2, a=x, epi=step.EPI_GELU_MUL, rowmap=step.ROWS_GATE_UP, out=mid, table=table)
    prog.finalize().launch(prog.io())
    gu = oracle.t16_gemv(u16(x), *_np(qs, d), 1, 2)
    assert np.array_equal(u16(table), oracle.gelu_table())
    assert np.array_equal(u16(mid), oracle.gelu_mul(gu[:i], gu[i:], oracle.gelu_table()))
    ab = gu[:i] & 0x7FFF
    assert (ab < 0x3B00).any() and ((ab >= 0x3B00) & (ab < 0x4300)).any() and (ab >= 0x4300).any()


@pytest.mark.parametrize("rot,pos_v", [(64, 777), (0, 4000)])
def test_qkv_stage_spark(cuda, oracle, rot, pos_v):
    """head_dim 256 with partial (64) or full rotary, gate rows -> sigmoid gate."""
    import torch
    from spark_b200 import step
    h = 2560
    n = (NQ + 2 * NKV) * D + 16
    qs, d = _q4(n, h, seed=21 + rot)
    w = step.q4_pack_t16(qs, d, 1, step.ROWS_PAIR_HALF, D, rot)
    kc, vc, table = _caches(4096, seed=5)
    kc0, vc0 = u16(kc), u16(vc)
    r = rot or D
    g = torch.Generator(device="cuda").manual_seed(7)
    cs = (torch.rand((4096 + 8, r), generator=g, device="cuda") * 2 - 1).to(torch.bfloat16)
    pos = torch.tensor([pos_v], device="cuda", dtype=torch.int64)
    q = torch.empty((NQ, D), device="cuda", dtype=torch.bfloat16)
    kv_new = torch.empty((2, NKV, D), device="cuda", dtype=torch.bfloat16)
    gate = torch.empty(NQ, device="cuda", dtype=torch.bfloat16)
    a = torch.randn(h, device="cuda").to(torch.bfloat16)
    gamma = (1 + 0.02 * torch.randn(h, device="cuda")).to(torch.bfloat16)
    res = torch.empty(h, device="cuda", dtype=torch.bfloat16)
    rope = {"cos_sin": cs, "pos": pos, "block_table": table, "k_cache": kc, "v_cache": vc, "q": q,
            "kv_new": kv_new, "block_size": BS, "nq": NQ, "nkv": NKV}
    prog = step.StepProgram("cuda")
    prog.gemv(w, n, h, ks=4, a=a, gamma=gamma, eps=1e-6, res_out=res, epi=step.EPI_ROPE_KV,
              rowmap=step.ROWS_PAIR_HALF, head_dim=D, rope=rope, rotary_dim=rot, gate=gate)
    prog.finalize().launch(prog.io())
    torch.cuda.synchronize()
    _, xn = oracle.add_rmsnorm(u16(a), None, u16(gamma), 1e-6)
    y = oracle.t16_gemv(xn, *_np(qs, d), 1, 4)
    qkv = y[:(NQ + 2 * NKV) * D].reshape(NQ + 2 * NKV, D)
    rotd = oracle.rope_partial(qkv[:NQ + NKV], r, u16(cs)[pos_v])
    assert np.array_equal(u16(q), rotd[:NQ])
    assert np.array_equal(u16(gate), oracle.sigmoid_bf16(y[(NQ + 2 * NKV) * D:(NQ + 2 * NKV) * D + NQ]))
    blk, off = int(table[pos_v // BS].item()), pos_v % BS
    kc1, vc1 = u16(kc), u16(vc)
    assert np.array_equal(kc1[blk, :, off], rotd[NQ:])
    assert np.array_equal(vc1[blk, :, off], qkv[NQ + NKV:])
    assert np.array_equal(u16(kv_new)[0], rotd[NQ:]) and np.array_equal(u16(kv_new)[1], qkv[NQ + NKV:])
    kc1[blk, :, off] = kc0[blk, :, off]
    vc1[blk, :, off] = vc0[blk, :, off]
    assert np.array_equal(kc1, kc0) and np.array_equal(vc1, vc0)


# 37 splits x 4 kv heads = 148 tasks (one per CTA); 74 splits: two per CTA.  Windows
# whose start is not a multiple of 16 (masked positions at the head of split 0).
@pytest.mark.parametrize("L,splits,window,gated", [(1, 37, 0, True), (300, 37, 0, False), (2048, 37, 0, True),
                                                   (5000, 37, 513, True), (700, 37, 512, False),
                                                   (513, 37, 513, True), (9000, 74, 0, True),
                                                   (20000, 74, 513, True)])
def test_attention_stage_spark(cuda, oracle, L, splits, window, gated):
    import torch
    from spark_b200 import step
    kc, vc, table = _caches(L, seed=L + window)
    pos_v = L - 1
    blk, off = int(table[pos_v // BS].item()), pos_v % BS
    kv_new = torch.stack([kc[blk, :, off], vc[blk, :, off]]).contiguous()
    g = torch.Generator(device="cuda").manual_seed(L + 1)
    q = torch.randn((NQ, D), generator=g, device="cuda").to(torch.bfloat16)
    gate = torch.rand(NQ, generator=g, device="cuda").to(torch.bfloat16) if gated else None
    pos = torch.tensor([pos_v], device="cuda", dtype=torch.int64)
    po = torch.empty((splits, NQ, D), device="cuda", dtype=torch.float32)
    pl = torch.empty((splits, NQ), device="cuda", dtype=torch.float32)
    out = torch.empty((NQ, D), device="cuda", dtype=torch.bfloat16)
    hc = torch.zeros(NKV, device="cuda", dtype=torch.int32)
    T = step.max_split_tokens(min(L, window + 16) if window else L, splits)
    scale = float(np.float32(1 / math.sqrt(D)))
    prog = step.StepProgram("cuda")
    prog.attention(q=q, k_cache=kc, v_cache=vc, kv_new=kv_new, block_table=table, pos=pos, splits=splits,
                   max_split_tokens=T, scale=scale, part_o=po, part_lse=pl, head_counters=hc, attn_out=out, nq=NQ,
                   nkv=NKV, head_dim=D, block_size=BS, window=window, gate=gate)
    prog.finalize().launch(prog.io())
    torch.cuda.synchronize()
    wpo, wpl = oracle.attn_split(u16(q), u16(kc), u16(vc), table.cpu().numpy(), L, splits, scale,
                                 chunk_accs=step.CHUNK_ACCS, window=window)
    assert np.array_equal(pl.cpu().numpy().view(np.uint32), wpl.view(np.uint32))
    assert np.array_equal(po.cpu().numpy().view(np.uint32), wpo.view(np.uint32))
    want = oracle.attn_combine(wpo, wpl, None if gate is None else u16(gate))
    assert np.array_equal(u16(out), want)
    assert bool((hc == splits).all())


def test_spark_attention_needs_head_dim_256(cuda):
    """The Spark instantiation's attention is head_dim 256: a window on a 128-dim head is refused."""
    import torch
    from spark_b200 import step
    from spark_b200._lib import SparkError
    nq, nkv, d = 32, 8, 128
    kc = torch.zeros((4, nkv, BS, d), device="cuda", dtype=torch.bfloat16)

    def z(*s, dt=torch.float32):
        return torch.zeros(s, device="cuda", dtype=dt)

    prog = step.StepProgram("cuda")
    prog.attention(q=z(nq, d, dt=torch.bfloat16), k_cache=kc, v_cache=kc, kv_new=z(2, nkv, d, dt=torch.bfloat16),
                   block_table=z(4, dt=torch.int32), pos=z(1, dt=torch.int64), splits=18, max_split_tokens=64,
                   scale=0.1, part_o=z(18, nq, d), part_lse=z(18, nq), head_counters=z(nkv, dt=torch.int32),
                   attn_out=z(nq, d, dt=torch.bfloat16), nq=nq, nkv=nkv, head_dim=d, block_size=BS, window=512)
    with pytest.raises(SparkError):
        prog.finalize().launch(prog.io())
