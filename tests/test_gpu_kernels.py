"""GPU parity of every sm_100a kernel against the CPU oracle (bit-exact) and, for the
GEMV and attention, against float64 dequantize-then-matmul / eager attention within
the north-star tolerances (GEMV rel 1e-2 / abs 1e-3, attention abs 2e-2).

All calls go through the C ABI (spark_b200.ops -> libspark_b200.so)."""
from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _t():
    import torch
    return torch


def u16(t):
    torch = _t()
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def dev_bf16(a, device):
    torch = _t()
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16)).view(torch.bfloat16).to(device)


def dev_f16(a, device):
    torch = _t()
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16)).view(torch.float16).to(device)


def rand_q4(oracle, n, k, seed, std=0.02):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * std).astype(np.float32)
    qs, d = oracle.q4_quantize(w)
    return qs, d


# ----------------------------------------------------------------------------- Q4_0 format kernels
def test_quantize_kernel_matches_gguf_golden(cuda, oracle):
    torch = _t()
    from spark_b200 import ops
    z = np.load(GOLDEN / "q4_0_gguf.npz")
    for n in sorted({k.split(".")[0] for k in z.files}):
        w = torch.from_numpy(z[n + ".w"]).to(cuda)
        qs, d = ops.q4_quantize(w)
        torch.cuda.synchronize()
        got = oracle.q4_join(qs.cpu().numpy(), u16(d))
        assert np.array_equal(got.reshape(-1), z[n + ".blocks"].reshape(-1)), n


def test_quantize_kernel_matches_oracle_large(cuda, oracle):
    torch = _t()
    from spark_b200 import ops
    g = torch.Generator(device=cuda).manual_seed(7)
    w = torch.randn((1024, 2560), generator=g, device=cuda) * 0.02
    qs, d = ops.q4_quantize(w)
    oqs, od = oracle.q4_quantize(w.cpu().numpy())
    assert np.array_equal(qs.cpu().numpy(), oqs) and np.array_equal(u16(d), od)


def test_split_and_dequant_kernels(cuda, oracle):
    torch = _t()
    from spark_b200 import ops
    z = np.load(GOLDEN / "q4_0_gguf.npz")
    blocks, w = z["normal.blocks"], z["normal.w"]
    qs, d = ops.q4_split_gguf(torch.from_numpy(blocks.reshape(-1).copy()).to(cuda), w.shape[0], w.shape[1])
    oqs, od = oracle.q4_split(blocks, w.shape[0], w.shape[1])
    assert np.array_equal(qs.cpu().numpy(), oqs) and np.array_equal(u16(d), od)
    deq = ops.q4_dequantize(qs, d)
    assert np.array_equal(u16(deq), oracle.f32_to_bf16(oracle.q4_dequantize(oqs, od)))


# ----------------------------------------------------------------------------- GEMV
GEMV_SHAPES = [
    (9728, 2560, 1),    # BASELINE config 0 (single-op GEMV)
    (6144, 2560, 1),    # qkv
    (2560, 4096, 1),    # o_proj
    (19456, 2560, 1),   # gate_up
    (2560, 9728, 1),    # down
    (256, 256, 1),      # tiny
    (98, 544, 1),       # K/32 = 17: uneven blocks per lane
    (2, 32, 1),         # one block
    (640, 2560, 2),
    (512, 1024, 3),
    (256, 4096, 8),
]


@pytest.fixture(params=["ring", "direct"])
def gemv_path(request, cuda):
    """Run a GEMV test through both implementations (they must agree bit for bit)."""
    from spark_b200 import ops
    ops.set_gemv_ring(request.param == "ring")
    ops.read_device_error(reset=True)
    yield request.param
    assert ops.read_device_error(reset=True) == 0, "a bounded wait timed out"
    ops.set_gemv_ring(True)


@pytest.mark.parametrize("n,k,batch", GEMV_SHAPES)
def test_q4_gemv_bit_exact(cuda, oracle, gemv_path, n, k, batch):
    torch = _t()
    from spark_b200 import ops
    qs, d = rand_q4(oracle, n, k, seed=n + k)
    rng = np.random.default_rng(batch)
    x = oracle.f32_to_bf16(rng.standard_normal((batch, k)).astype(np.float32))
    y = ops.q4_gemv(dev_bf16(x, cuda), torch.from_numpy(qs).to(cuda), dev_f16(d, cuda))
    torch.cuda.synchronize()
    got = u16(y).reshape(batch, n)
    exp = oracle.q4_gemv(x, qs, d)
    assert np.array_equal(got, exp), f"{np.count_nonzero(got != exp)} of {got.size} differ"
    # reference PyTorch path: dequantize -> matmul
    wf = torch.from_numpy(oracle.q4_dequantize(qs, d)).double()
    ref = (torch.from_numpy(oracle.bf16_to_f32(x)).double() @ wf.T).numpy()
    yf = oracle.bf16_to_f32(got)
    assert np.all(np.abs(yf - ref) <= 1e-3 + 1e-2 * np.abs(ref))


def test_q4_gemv_rejects_bad_args(cuda):
    torch = _t()
    from spark_b200 import _lib, ops
    qs = torch.zeros((4, 16), dtype=torch.uint8, device=cuda)
    d = torch.zeros((4, 1), dtype=torch.float16, device=cuda)
    with pytest.raises(ValueError):
        ops.q4_gemv(torch.zeros(32, dtype=torch.float32, device=cuda), qs, d)
    with pytest.raises(_lib.SparkError):
        _lib.call("spark_q4_gemv", None, None, None, None, 4, 32, 1, None)


def _norm_inputs(oracle, k, seed):
    rng = np.random.default_rng(seed)
    a = oracle.f32_to_bf16(rng.standard_normal(k).astype(np.float32))
    b = oracle.f32_to_bf16(rng.standard_normal(k).astype(np.float32))
    g = oracle.f32_to_bf16((1 + 0.02 * rng.standard_normal(k)).astype(np.float32))
    return a, b, g


@pytest.mark.parametrize("with_b", [True, False])
def test_rmsnorm_q4_gemv_bit_exact(cuda, oracle, gemv_path, with_b):
    torch = _t()
    from spark_b200 import ops
    n, k, eps = 2048, 2560, 1e-6
    qs, d = rand_q4(oracle, n, k, seed=11)
    a, b, g = _norm_inputs(oracle, k, 12)
    res_dev = torch.empty(k, dtype=torch.bfloat16, device=cuda)
    y = torch.empty(n, dtype=torch.bfloat16, device=cuda)
    ops.rmsnorm_q4_gemv_out(dev_bf16(a, cuda), dev_bf16(b, cuda) if with_b else None, dev_bf16(g, cuda), eps,
                            torch.from_numpy(qs).to(cuda), dev_f16(d, cuda), y, res_dev)
    torch.cuda.synchronize()
    res, x = oracle.add_rmsnorm(a, b if with_b else None, g, eps)
    assert np.array_equal(u16(res_dev), res)
    assert np.array_equal(u16(y), oracle.q4_gemv(x, qs, d)[0])


def test_gate_up_silu_bit_exact(cuda, oracle, gemv_path):
    torch = _t()
    from spark_b200 import ops
    inter, k, eps = 1536, 2560, 1e-6
    qs, d = rand_q4(oracle, 2 * inter, k, seed=21)
    a, b, g = _norm_inputs(oracle, k, 22)
    mid = torch.empty(inter, dtype=torch.bfloat16, device=cuda)
    res_dev = torch.empty(k, dtype=torch.bfloat16, device=cuda)
    ops.rmsnorm_gate_up_silu_out(dev_bf16(a, cuda), dev_bf16(b, cuda), dev_bf16(g, cuda), eps,
                                 torch.from_numpy(qs).to(cuda), dev_f16(d, cuda), mid, res_dev)
    torch.cuda.synchronize()
    res, x = oracle.add_rmsnorm(a, b, g, eps)
    gu = oracle.q4_gemv(x, qs, d)[0]
    assert np.array_equal(u16(res_dev), res)
    assert np.array_equal(u16(mid), oracle.silu_mul(gu[:inter], gu[inter:]))


@pytest.mark.parametrize("pos,use_slot_mapping", [(0, False), (777, False), (4095, True)])
def test_qkv_rope_kvstore_bit_exact(cuda, oracle, gemv_path, pos, use_slot_mapping):
    torch = _t()
    from spark_b200 import ops
    from spark_b200.config import SparkConfig
    from spark_b200.model import rope_cos_sin
    cfg = SparkConfig(max_position=8192)
    nq, nkv, D, k, bs, eps = 32, 8, 128, 2560, 128, 1e-6
    qs, d = rand_q4(oracle, (nq + 2 * nkv) * D, k, seed=31)
    a, b, g = _norm_inputs(oracle, k, 32)
    cs = rope_cos_sin(cfg)
    cs_np = u16(cs)
    pool = 64
    rng = np.random.default_rng(pos)
    table = rng.permutation(pool)[:pool // 2].astype(np.int32)
    kc = torch.zeros((pool, nkv, bs, D), dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    q = torch.empty((nq, D), dtype=torch.bfloat16, device=cuda)
    res_dev = torch.empty(k, dtype=torch.bfloat16, device=cuda)
    pos_t = torch.tensor([pos], dtype=torch.int64, device=cuda)
    slot = int(table[pos // bs]) * bs + pos % bs
    slot_t = torch.tensor([slot], dtype=torch.int64, device=cuda) if use_slot_mapping else None
    ops.qkv_rope_kvstore_out(dev_bf16(a, cuda), dev_bf16(b, cuda), dev_bf16(g, cuda), eps,
                             torch.from_numpy(qs).to(cuda), dev_f16(d, cuda), nq, nkv, D, cs.to(cuda), pos_t,
                             torch.from_numpy(table).to(cuda), slot_t, bs, kc, vc, q, res_dev)
    torch.cuda.synchronize()
    res, x = oracle.add_rmsnorm(a, b, g, eps)
    qkv = oracle.q4_gemv(x, qs, d)[0].reshape(nq + 2 * nkv, D)
    rot = oracle.rope_neox(qkv[:nq + nkv], cs_np[pos])
    assert np.array_equal(u16(res_dev), res)
    assert np.array_equal(u16(q), rot[:nq])
    blk, off = slot // bs, slot % bs
    kc_np, vc_np = u16(kc), u16(vc)
    assert np.array_equal(kc_np[blk, :, off], rot[nq:])
    assert np.array_equal(vc_np[blk, :, off], qkv[nq + nkv:])
    kc_np[blk, :, off] = 0
    vc_np[blk, :, off] = 0
    assert not kc_np.any() and not vc_np.any(), "store touched other slots"


def test_qkv_embedding_input(cuda, oracle):
    """Layer 0 reads its input row straight from the embedding table."""
    torch = _t()
    from spark_b200 import ops
    from spark_b200.config import SparkConfig
    from spark_b200.model import rope_cos_sin
    cfg = SparkConfig(max_position=256)
    nq, nkv, D, k, bs, eps = 8, 2, 128, 512, 128, 1e-6
    qs, d = rand_q4(oracle, (nq + 2 * nkv) * D, k, seed=41)
    rng = np.random.default_rng(42)
    emb = oracle.f32_to_bf16((rng.standard_normal((50, k)) * 0.02).astype(np.float32))
    g = oracle.f32_to_bf16(np.ones(k, np.float32))
    cs = rope_cos_sin(SparkConfig(hidden_size=k, num_q_heads=nq, num_kv_heads=nkv, max_position=256))
    kc = torch.zeros((4, nkv, bs, D), dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    q = torch.empty((nq, D), dtype=torch.bfloat16, device=cuda)
    res = torch.empty(k, dtype=torch.bfloat16, device=cuda)
    tok = torch.tensor([37], dtype=torch.int32, device=cuda)
    ops.qkv_rope_kvstore_out(None, None, dev_bf16(g, cuda), eps, torch.from_numpy(qs).to(cuda), dev_f16(d, cuda),
                             nq, nkv, D, cs.to(cuda), torch.tensor([5], dtype=torch.int64, device=cuda),
                             torch.tensor([2, 0], dtype=torch.int32, device=cuda), None, bs, kc, vc, q, res,
                             embed=dev_bf16(emb, cuda), token=tok)
    torch.cuda.synchronize()
    r, x = oracle.add_rmsnorm(emb[37], None, g, eps)
    assert np.array_equal(u16(res), emb[37])
    qkv = oracle.q4_gemv(x, qs, d)[0].reshape(nq + 2 * nkv, D)
    assert np.array_equal(u16(q), oracle.rope_neox(qkv[:nq + nkv], u16(cs)[5])[:nq])


def test_head_argmax_bit_exact(cuda, oracle, gemv_path):
    torch = _t()
    from spark_b200 import ops
    n, k, eps = 151936, 2560, 1e-6
    qs, d = rand_q4(oracle, n, k, seed=51)
    a, b, g = _norm_inputs(oracle, k, 52)
    logits = torch.empty(n, dtype=torch.bfloat16, device=cuda)
    key = torch.zeros(1, dtype=torch.int64, device=cuda)
    ops.head_argmax_out(dev_bf16(a, cuda), dev_bf16(b, cuda), dev_bf16(g, cuda), eps,
                        torch.from_numpy(qs).to(cuda), dev_f16(d, cuda), logits, key)
    tok = torch.zeros(1, dtype=torch.int32, device=cuda)
    ops.decode_finalize(key, tok)
    torch.cuda.synchronize()
    _, x = oracle.add_rmsnorm(a, b, g, eps)
    exp = oracle.q4_gemv(x, qs, d)[0]
    assert np.array_equal(u16(logits), exp)
    assert int(tok.item()) == oracle.argmax_bf16(exp)
    assert int(key.item()) == 0, "finalize must reset the argmax key"


def test_argmax_ties_pick_lowest_index(cuda, oracle):
    """All-zero head weights make every logit 0: the argmax must be index 0."""
    torch = _t()
    from spark_b200 import ops
    n, k = 4096, 256
    qs = torch.full((n, k // 2), 0x88, dtype=torch.uint8, device=cuda)  # q = 8 -> weight 0
    d = torch.ones((n, k // 32), dtype=torch.float16, device=cuda)
    a = torch.randn(k, device=cuda).to(torch.bfloat16)
    g = torch.ones(k, dtype=torch.bfloat16, device=cuda)
    logits = torch.empty(n, dtype=torch.bfloat16, device=cuda)
    key = torch.zeros(1, dtype=torch.int64, device=cuda)
    ops.head_argmax_out(a, None, g, 1e-6, qs, d, logits, key)
    tok = torch.zeros(1, dtype=torch.int32, device=cuda)
    ops.decode_finalize(key, tok)
    torch.cuda.synchronize()
    assert int(tok.item()) == 0


# ----------------------------------------------------------------------------- attention
def _paged_cache(oracle, rng, L, nkv=8, D=128, bs=128, pool_factor=4):
    nblk = max(1, (L + bs - 1) // bs)
    pool = nblk * pool_factor
    kc = oracle.f32_to_bf16(rng.standard_normal((pool, nkv, bs, D)).astype(np.float32))
    vc = oracle.f32_to_bf16(rng.standard_normal((pool, nkv, bs, D)).astype(np.float32))
    table = rng.permutation(pool)[:nblk].astype(np.int32)
    return kc, vc, table


@pytest.mark.parametrize("L,splits", [(1, 16), (17, 16), (129, 16), (2048, 16), (4096, 16), (6144, 16),
                                      (1000, 3), (300, 64), (32768, 64)])
def test_attention_bit_exact(cuda, oracle, L, splits):
    torch = _t()
    from spark_b200 import ops
    rng = np.random.default_rng(L * 7 + splits)
    kc, vc, table = _paged_cache(oracle, rng, L)
    nq, D = 32, 128
    q = oracle.f32_to_bf16(rng.standard_normal((nq, D)).astype(np.float32))
    scale = float(np.float32(1 / math.sqrt(D)))
    T = oracle.split_tokens(L, splits)
    po = torch.empty((splits, nq, D), dtype=torch.float32, device=cuda)
    pl = torch.empty((splits, nq), dtype=torch.float32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    ops.attn_splitkv_out(dev_bf16(q, cuda), dev_bf16(kc, cuda), dev_bf16(vc, cuda), torch.from_numpy(table).to(cuda),
                         splits, T, scale, po, pl, pos=torch.tensor([L - 1], dtype=torch.int64, device=cuda),
                         error=err)
    out = torch.empty((nq, D), dtype=torch.bfloat16, device=cuda)
    ops.attn_combine_out(po, pl, out)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    epo, epl = oracle.attn_split(q, kc, vc, table, L, splits, scale)
    assert np.array_equal(pl.cpu().numpy().view(np.uint32), epl.view(np.uint32))
    assert np.array_equal(po.cpu().numpy().view(np.uint32), epo.view(np.uint32))
    eout = oracle.attn_combine(epo, epl)
    assert np.array_equal(u16(out), eout)
    # eager float64 attention (the reference's PyTorch path)
    t = np.arange(L)
    blk, off = table[t // 128], t % 128
    ref = np.zeros((nq, D))
    for h in range(nq):
        K = oracle.bf16_to_f32(kc[blk, h // 4, off]).astype(np.float64)
        V = oracle.bf16_to_f32(vc[blk, h // 4, off]).astype(np.float64)
        s = K @ oracle.bf16_to_f32(q[h]).astype(np.float64) * scale
        p = np.exp(s - s.max())
        ref[h] = p @ V / p.sum()
    assert np.max(np.abs(oracle.bf16_to_f32(u16(out)) - ref)) < 2e-2


@pytest.mark.parametrize("L,splits", [(1, 16), (130, 16), (2048, 48), (6144, 48), (5000, 3), (700, 256)])
def test_attention_fused_decode_bit_exact(cuda, oracle, L, splits):
    """Split + fused combine == oracle split + combine, twice in a row (counters self-reset)."""
    torch = _t()
    from spark_b200 import ops
    rng = np.random.default_rng(L + 31 * splits)
    kc, vc, table = _paged_cache(oracle, rng, L)
    nq, D = 32, 128
    scale = float(np.float32(1 / math.sqrt(D)))
    T = oracle.split_tokens(L, splits)
    po = torch.empty((splits, nq, D), dtype=torch.float32, device=cuda)
    pl = torch.empty((splits, nq), dtype=torch.float32, device=cuda)
    counters = torch.zeros(8, dtype=torch.int32, device=cuda)
    out = torch.empty((nq, D), dtype=torch.bfloat16, device=cuda)
    kd, vd, td = dev_bf16(kc, cuda), dev_bf16(vc, cuda), torch.from_numpy(table).to(cuda)
    for rep in range(2):
        q = oracle.f32_to_bf16(rng.standard_normal((nq, D)).astype(np.float32))
        ops.attn_decode_out(dev_bf16(q, cuda), kd, vd, td, splits, T, scale, po, pl, counters, out,
                            pos=torch.tensor([L - 1], dtype=torch.int64, device=cuda))
        torch.cuda.synchronize()
        epo, epl = oracle.attn_split(q, kc, vc, table, L, splits, scale)
        assert np.array_equal(u16(out), oracle.attn_combine(epo, epl)), rep
        assert np.array_equal(pl.cpu().numpy().view(np.uint32), epl.view(np.uint32))
        assert int(counters.abs().sum().item()) == 0


def test_attention_seq_len_input_and_overflow_flag(cuda, oracle):
    torch = _t()
    from spark_b200 import ops
    rng = np.random.default_rng(3)
    L, splits = 600, 4
    kc, vc, table = _paged_cache(oracle, rng, L)
    q = oracle.f32_to_bf16(rng.standard_normal((32, 128)).astype(np.float32))
    scale = float(np.float32(1 / math.sqrt(128)))
    po = torch.empty((splits, 32, 128), dtype=torch.float32, device=cuda)
    pl = torch.empty((splits, 32), dtype=torch.float32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    args = (dev_bf16(q, cuda), dev_bf16(kc, cuda), dev_bf16(vc, cuda), torch.from_numpy(table).to(cuda), splits)
    ops.attn_splitkv_out(*args, 160, scale, po, pl, seq_len=torch.tensor([L], dtype=torch.int32, device=cuda),
                         error=err)
    torch.cuda.synchronize()
    epo, epl = oracle.attn_split(q, kc, vc, table, L, splits, scale)
    assert int(err.item()) == 0 and np.array_equal(po.cpu().numpy(), epo)
    # a split longer than the allocation is reported, not overrun
    ops.attn_splitkv_out(*args, 64, scale, po, pl, seq_len=torch.tensor([L], dtype=torch.int32, device=cuda),
                         error=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 1
    assert torch.isneginf(pl).all()


# ----------------------------------------------------------------------------- small kernels
def test_standalone_norm_silu_rope(cuda, oracle):
    torch = _t()
    from spark_b200 import ops
    from spark_b200.config import SparkConfig
    from spark_b200.model import rope_cos_sin
    a, b, g = _norm_inputs(oracle, 2560, 61)
    y = torch.empty(2560, dtype=torch.bfloat16, device=cuda)
    res = torch.empty_like(y)
    ops.add_rmsnorm_out(dev_bf16(a, cuda), dev_bf16(b, cuda), dev_bf16(g, cuda), 1e-6, y, res)
    er, ey = oracle.add_rmsnorm(a, b, g, 1e-6)
    rng = np.random.default_rng(62)
    gg = oracle.f32_to_bf16((rng.standard_normal(9728) * 4).astype(np.float32))
    uu = oracle.f32_to_bf16(rng.standard_normal(9728).astype(np.float32))
    m = torch.empty(9728, dtype=torch.bfloat16, device=cuda)
    ops.silu_mul_out(dev_bf16(gg, cuda), dev_bf16(uu, cuda), m)
    cs = rope_cos_sin(SparkConfig(max_position=2048))
    x = oracle.f32_to_bf16(rng.standard_normal((40, 128)).astype(np.float32))
    xd = dev_bf16(x, cuda)
    ops.rope_neox_(xd, cs.to(cuda), torch.tensor([1234], dtype=torch.int64, device=cuda))
    torch.cuda.synchronize()
    assert np.array_equal(u16(y), ey) and np.array_equal(u16(res), er)
    assert np.array_equal(u16(m), oracle.silu_mul(gg, uu))
    assert np.array_equal(u16(xd), oracle.rope_neox(x, u16(cs)[1234]))


def test_slot_mapping_kat_gpu(cuda, oracle):
    """tools/validation/test_slot_mapping.py cases, including graph replay with new positions."""
    torch = _t()
    from spark_b200 import ops
    z = np.load(GOLDEN / "slot_mapping_kat.npz")
    maximum = int(z["maximum"])
    tables = [torch.from_numpy(t.copy()).to(cuda) for t in z["tables"]]
    outs = [torch.full((maximum,), -99, dtype=torch.int64, device=cuda) for _ in z["sizes"]]
    for ci, (count, offset) in enumerate(z["cases"][:5]):
        pos = (torch.arange(int(count), dtype=torch.int64) + int(offset)).to(cuda)
        qsl = torch.tensor([0, int(count)], dtype=torch.int32, device=cuda)
        for gi, size in enumerate(z["sizes"]):
            ops.slot_mapping_out(int(count), qsl, pos if count else None, tables[gi], int(size), outs[gi])
        torch.cuda.synchronize()
        for gi in range(4):
            o = outs[gi].cpu().numpy()
            assert np.array_equal(o[:count], z[f"case{ci}.group{gi}"]) and np.all(o[count:] == -1)
    pos = torch.tensor([4095], dtype=torch.int64, device=cuda)
    qsl = torch.tensor([0, 1], dtype=torch.int32, device=cuda)
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for gi, size in enumerate(z["sizes"]):
            ops.slot_mapping_out(1, qsl, pos, tables[gi], int(size), outs[gi])
    torch.cuda.synchronize()
    with torch.cuda.graph(graph):
        for gi, size in enumerate(z["sizes"]):
            ops.slot_mapping_out(1, qsl, pos, tables[gi], int(size), outs[gi])
    for ci, offset in zip((5, 6, 7), (4096, 127, 8192)):
        pos.fill_(offset)
        graph.replay()
        torch.cuda.synchronize()
        for gi in range(4):
            o = outs[gi].cpu().numpy()
            assert o[0] == z[f"case{ci}.group{gi}"][0] and np.all(o[1:] == -1)
