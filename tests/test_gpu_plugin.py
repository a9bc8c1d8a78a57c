"""GPU parity of the vLLM plugin classes (the drop-in boundary): the spark_q4_0 linear
method, the attention backend's decode / prefill paths and the Q6_K LM head method,
against the oracle."""
from __future__ import annotations

import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

vllm = pytest.importorskip("vllm")


def u16(t):
    import torch
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def test_q4_linear_method_loads_gguf_blocks_and_matches_oracle(cuda, oracle):
    import torch
    from spark_b200.plugin.quant import SparkQ4Config, SparkQ4LinearMethod
    rng = np.random.default_rng(4)
    n, k = 1024, 2560
    qs, d = oracle.q4_quantize((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    blocks = oracle.q4_join(qs, d)
    method = SparkQ4LinearMethod(SparkQ4Config())
    layer = torch.nn.Module()
    method.create_weights(layer, k, [n // 2, n // 2], k, n, torch.bfloat16)
    layer.qweight.data = torch.from_numpy(blocks).cuda()
    method.process_weights_after_loading(layer)
    assert np.array_equal(layer.qs.cpu().numpy(), qs) and np.array_equal(u16(layer.d), d)
    for rows in (1, 3):  # decode: fused Q4_0 GEMV
        x = torch.randn((rows, k), device="cuda").to(torch.bfloat16)
        y = method.apply(layer, x)
        assert y.shape == (rows, n)
        assert np.array_equal(u16(y), oracle.q4_gemv(u16(x), qs, d))
    x = torch.randn((20, k), device="cuda").to(torch.bfloat16)  # prefill: dequantize + bf16 matmul
    bias = torch.randn(n, device="cuda").to(torch.bfloat16)
    y = method.apply(layer, x, bias).float().cpu().numpy()
    ref = oracle.bf16_to_f32(u16(x)).astype(np.float64) @ oracle.q4_dequantize(qs, d).astype(np.float64).T
    ref += oracle.bf16_to_f32(u16(bias))
    assert np.max(np.abs(y - ref)) <= 2e-2 * np.abs(ref).max()


def _backend_setup(seq_lens, nq=32, nkv=8, D=128, bs=128, seed=0):
    import torch
    from spark_b200.plugin.attention import SparkAttentionImpl, SparkAttentionMetadata
    g = torch.Generator(device="cuda").manual_seed(seed)
    nblk = sum(-(-n // bs) for n in seq_lens) + 3
    kv = torch.randn((2, nblk, nkv, bs, D), generator=g, device="cuda").to(torch.bfloat16)
    perm = torch.randperm(nblk, generator=g, device="cuda").to(torch.int32)
    maxb = max(-(-n // bs) for n in seq_lens)
    table = torch.zeros((len(seq_lens), maxb), dtype=torch.int32, device="cuda")
    off = 0
    for r, n in enumerate(seq_lens):
        nb = -(-n // bs)
        table[r, :nb] = perm[off:off + nb]
        off += nb
    impl = SparkAttentionImpl(nq, D, 1 / math.sqrt(D), nkv)
    return kv, table, impl, SparkAttentionMetadata


def test_attention_backend_decode_matches_oracle(cuda, oracle):
    import torch
    nq, nkv, D, bs = 32, 8, 128, 128
    seq_lens = [300, 2049]
    kv, table, impl, MD = _backend_setup(seq_lens)
    t = len(seq_lens)
    q = torch.randn((t, nq * D), device="cuda").to(torch.bfloat16)
    k = torch.randn((t, nkv * D), device="cuda").to(torch.bfloat16)
    v = torch.randn((t, nkv * D), device="cuda").to(torch.bfloat16)
    slots = torch.tensor([int(table[r, (n - 1) // bs]) * bs + (n - 1) % bs for r, n in enumerate(seq_lens)],
                         device="cuda", dtype=torch.int64)
    md = MD(num_actual_tokens=t, num_reqs=t, max_query_len=1, max_seq_len=max(seq_lens),
            query_start_loc=torch.arange(t + 1, device="cuda", dtype=torch.int32),
            query_start_loc_cpu=torch.arange(t + 1, dtype=torch.int32),
            seq_lens=torch.tensor(seq_lens, device="cuda", dtype=torch.int32), block_table=table, slot_mapping=slots,
            splits=24, max_split_tokens=96)
    out = torch.empty((t, nq * D), device="cuda", dtype=torch.bfloat16)
    impl.forward(None, q, k, v, kv, md, out)
    torch.cuda.synchronize()
    kc, vc = u16(kv[0]), u16(kv[1])
    for r, n in enumerate(seq_lens):  # this step's k / v landed at the slot
        blk, o = int(table[r, (n - 1) // bs]), (n - 1) % bs
        assert np.array_equal(kc[blk, :, o], u16(k[r]).reshape(nkv, D))
        assert np.array_equal(vc[blk, :, o], u16(v[r]).reshape(nkv, D))
        po, pl = oracle.attn_split(u16(q[r]).reshape(nq, D), kc, vc, table[r].cpu().numpy(), n, 24, impl.scale)
        assert np.array_equal(u16(out[r]).reshape(nq, D), oracle.attn_combine(po, pl))


def test_attention_backend_spark_head256_window(cuda, oracle):
    """The Spark model's attention through the vLLM backend: head_size 256, 16 q / 4 kv
    heads, a sliding layer (window 512 -> the reference's 513 positions) and a full one;
    decode bit-exact against the oracle's persistent-step order, twice in a row."""
    import torch
    from spark_b200 import step
    nq, nkv, D, bs = 16, 4, 256, 128
    seq_lens = [300, 2049]
    for window in (None, 512):
        kv, table, _, MD = _backend_setup(seq_lens, nq=nq, nkv=nkv, D=D, seed=7)
        from spark_b200.plugin.attention import SparkAttentionImpl
        impl = SparkAttentionImpl(nq, D, 1 / 16, nkv, sliding_window=window)
        t = len(seq_lens)
        q = torch.randn((t, nq * D), device="cuda").to(torch.bfloat16)
        k = torch.randn((t, nkv * D), device="cuda").to(torch.bfloat16)
        v = torch.randn((t, nkv * D), device="cuda").to(torch.bfloat16)
        slots = torch.tensor([int(table[r, (n - 1) // bs]) * bs + (n - 1) % bs for r, n in enumerate(seq_lens)],
                             device="cuda", dtype=torch.int64)
        md = MD(num_actual_tokens=t, num_reqs=t, max_query_len=1, max_seq_len=max(seq_lens),
                query_start_loc=torch.arange(t + 1, device="cuda", dtype=torch.int32),
                query_start_loc_cpu=torch.arange(t + 1, dtype=torch.int32),
                seq_lens=torch.tensor(seq_lens, device="cuda", dtype=torch.int32), block_table=table,
                slot_mapping=slots, splits=24, max_split_tokens=96)
        out = torch.empty((t, nq * D), device="cuda", dtype=torch.bfloat16)
        for rep in range(2):  # a second call (next launch generation) gives the same
            impl.forward(None, q, k, v, kv, md, out)
            torch.cuda.synchronize()
            kc, vc = u16(kv[0]), u16(kv[1])
            for r, n in enumerate(seq_lens):
                S = impl._step["splits"]
                po, pl = oracle.attn_split(u16(q[r]).reshape(nq, D), kc, vc, table[r].cpu().numpy(), n, S,
                                           impl.scale, chunk_accs=step.CHUNK_ACCS, window=impl.window)
                assert np.array_equal(u16(out[r]).reshape(nq, D), oracle.attn_combine(po, pl)), (window, r, rep)
        assert int(impl._step["error"].item()) == 0


def test_attention_backend_prefill_causal(cuda, oracle):
    import torch
    nq, nkv, D, bs = 32, 8, 128, 128
    n, lq = 200, 5
    kv, table, impl, MD = _backend_setup([n], seed=3)
    q = torch.randn((lq, nq * D), device="cuda").to(torch.bfloat16)
    k = torch.randn((lq, nkv * D), device="cuda").to(torch.bfloat16)
    v = torch.randn((lq, nkv * D), device="cuda").to(torch.bfloat16)
    pos = list(range(n - lq, n))
    slots = torch.tensor([int(table[0, p // bs]) * bs + p % bs for p in pos], device="cuda", dtype=torch.int64)
    md = MD(num_actual_tokens=lq, num_reqs=1, max_query_len=lq, max_seq_len=n,
            query_start_loc=torch.tensor([0, lq], device="cuda", dtype=torch.int32),
            query_start_loc_cpu=torch.tensor([0, lq], dtype=torch.int32),
            seq_lens=torch.tensor([n], device="cuda", dtype=torch.int32), block_table=table, slot_mapping=slots,
            splits=16, max_split_tokens=16)
    out = torch.empty((lq, nq * D), device="cuda", dtype=torch.bfloat16)
    impl.forward(None, q, k, v, kv, md, out)
    torch.cuda.synchronize()
    kc = oracle.bf16_to_f32(u16(kv[0])).astype(np.float64)
    vc = oracle.bf16_to_f32(u16(kv[1])).astype(np.float64)
    qf = oracle.bf16_to_f32(u16(q)).astype(np.float64).reshape(lq, nq, D)
    got = oracle.bf16_to_f32(u16(out)).reshape(lq, nq, D)
    tb = table[0].cpu().numpy()
    for i in range(lq):
        L = pos[i] + 1
        for h in range(nq):
            hk = h // (nq // nkv)
            K = np.stack([kc[tb[t // bs], hk, t % bs] for t in range(L)])
            V = np.stack([vc[tb[t // bs], hk, t % bs] for t in range(L)])
            s = K @ qf[i, h] * impl.scale
            p = np.exp(s - s.max())
            ref = p @ V / p.sum()
            assert np.max(np.abs(got[i, h] - ref)) <= 2e-2


def test_q6_head_method_decode_matches_oracle(cuda, oracle):
    """The Q6_K LM head over a tied bf16 embedding (reference integration/head.py): one
    decode token runs the Q6_K GEMV bit-exactly in the oracle's order; other shapes take
    vLLM's bf16 path; a weight that is not the decode of the codes is refused."""
    import torch
    from spark_b200.plugin.head import install_q6_head
    rng = np.random.default_rng(6)
    vocab, hidden = 4096, 2560
    blocks = rng.integers(0, 256, size=(vocab * hidden // 256, 210), dtype=np.uint8)
    blocks[:, 208:210] = (rng.standard_normal(blocks.shape[0]) * 2e-5).astype(np.float16).view(np.uint8).reshape(-1, 2)
    weight = oracle.q6k_dequantize(blocks).reshape(vocab, hidden)
    head = torch.nn.Module()
    head.weight = torch.nn.Parameter(torch.from_numpy(weight).cuda().to(torch.bfloat16), requires_grad=False)
    tblocks = torch.from_numpy(blocks.reshape(vocab, -1)).cuda()
    bad = torch.nn.Module()
    bad.weight = torch.nn.Parameter(head.weight.detach().clone(), requires_grad=False)
    bad.weight.data[3, 7] += 1.0
    with pytest.raises(ValueError):
        install_q6_head(bad, tblocks)
    method = install_q6_head(head, tblocks)
    x = torch.randn((1, hidden), device="cuda").to(torch.bfloat16)
    for _ in range(2):  # the stage counters are left ready for the next call
        y = method.apply(head, x)
        assert y.shape == (1, vocab)
        want = oracle.parts_to_bf16(oracle.q6k_gemv_parts(u16(x), blocks.reshape(vocab, -1), vocab, hidden, 1, 4))
        assert np.array_equal(u16(y).reshape(-1), want)
    x2 = torch.randn((3, hidden), device="cuda").to(torch.bfloat16)
    y2 = method.apply(head, x2).float()
    ref = x2.float() @ head.weight.float().t()
    assert torch.allclose(y2, ref, rtol=2e-2, atol=2e-2)
