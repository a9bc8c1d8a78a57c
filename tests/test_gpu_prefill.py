"""Batched prefill (spark_b200.prefill: tensor-core GEMMs over the Q4_0 planes, or cuBLAS
over cached bf16 weights, + causal attention, the reference's standard prefill path) against token-by-token decode of the same prompt:
the paged K / V of every prompt position and the first token's logits agree within
bf16 rounding (not bit for bit: the GEMMs sum in their own order), for the synthetic
architecture and the Spark one (gate, GELU, sliding window shorter than the prompt,
partial RoPE, Q6_K head), with a prompt split over two chunks; decode continues from
the batched state."""
from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu


def _cfgs():
    from spark_b200.config import spark_x26_config, tiny_config
    return [tiny_config(num_layers=3),
            spark_x26_config(num_layers=4, hidden_size=512, num_q_heads=8, num_kv_heads=2, intermediate_size=1024,
                             vocab_size=4096, sliding_window=33, max_position=4096, name="spark-tiny")]


@pytest.mark.parametrize("gemm", ["q4", "bf16"])
@pytest.mark.parametrize("which", [0, 1])
def test_batched_prefill_matches_decode(cuda, which, gemm):
    import torch
    from spark_b200.model import DecodeEngine, SyntheticWeights
    cfg = _cfgs()[which]
    w = SyntheticWeights(cfg, device="cuda", seed=11)
    P = 90
    prompt = (torch.arange(P, dtype=torch.int32) * 131 + 7) % cfg.vocab_size
    ref = DecodeEngine(w, max_seq_len=256, num_blocks=8, seed=11)
    ref.prefill(prompt)
    torch.cuda.synchronize()
    eng = DecodeEngine(w, max_seq_len=256, num_blocks=8, seed=11)
    eng.prefill_batched(prompt, chunk=64, gemm=gemm)  # two chunks: the second attends to the first's cache
    torch.cuda.synchronize()
    bs = cfg.block_size
    pos = torch.arange(P, device="cuda")
    blk, off = eng.block_table[pos // bs].long(), pos % bs
    for li in range(cfg.num_layers):
        for c_ref, c in ((ref.k_cache[li], eng.k_cache[li]), (ref.v_cache[li], eng.v_cache[li])):
            a, b = c_ref[blk, :, off].float(), c[blk, :, off].float()
            assert (a - b).abs().max().item() <= 0.03 * a.abs().max().item() + 0.03, li
    lr, lg = ref.logits.float(), eng.logits.float()
    assert (lr - lg).abs().max().item() <= 0.03 * lr.abs().max().item() + 0.03
    assert int(eng.pos.item()) == P
    for _ in range(4):
        eng.step()
    torch.cuda.synchronize()
    assert int(eng.error.item()) == 0 and int(eng.pos.item()) == P + 4


def test_prefill_row_kernels(cuda, oracle):
    """spark_add_rmsnorm_rows against float64 (bf16 rounding), spark_rope_neox_rows bit for
    bit against the oracle's RoPE (the same products and rounding), partial rotary on a
    strided row view of a qkv output."""
    import numpy as np
    import torch
    from spark_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(5)
    n, h = 37, 2560
    a = torch.randn((n, h), generator=g, device="cuda").to(torch.bfloat16)
    b = torch.randn((n, h), generator=g, device="cuda").to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(h, generator=g, device="cuda")).to(torch.bfloat16)
    res, y = ops.add_rmsnorm_rows(a, b, gamma, 1e-6)
    s = a.double() + b.double()
    want = s * torch.rsqrt((s * s).mean(-1, keepdim=True) + 1e-6) * gamma.double()
    assert torch.equal(res, (a.float() + b.float()).to(torch.bfloat16))
    assert (y.double() - want).abs().max().item() <= 0.01 * want.abs().max().item()
    nh, D, rot, cols = 6, 256, 64, 6 * 256 + 16
    x = torch.randn((n, cols), generator=g, device="cuda").to(torch.bfloat16)
    cs = (torch.rand((n + 100, rot), generator=g, device="cuda") * 2 - 1).to(torch.bfloat16)
    x0 = x.clone()
    ops.rope_rows_(x, nh, D, rot, cs, 50)
    torch.cuda.synchronize()
    xs = x0.view(torch.int16).cpu().numpy().view(np.uint16)
    css = cs.view(torch.int16).cpu().numpy().view(np.uint16)
    got = x.view(torch.int16).cpu().numpy().view(np.uint16)
    for r in range(n):
        want_r = oracle.rope_partial(xs[r, :nh * D].reshape(nh, D), rot, css[50 + r])
        assert np.array_equal(got[r, :nh * D].reshape(nh, D), want_r), r
        assert np.array_equal(got[r, nh * D:], xs[r, nh * D:])  # the columns past the heads untouched


@pytest.mark.parametrize("i", [1024, 1020])  # 16-byte form, element form
def test_act_mul_rows_matches_decode_arithmetic(cuda, oracle, i):
    """spark_act_mul_rows: bit for bit the oracle's SiLU * mul and GELU-table * mul (the
    decode epilogues' arithmetic), over gate values spanning every range of the table."""
    import numpy as np
    import torch
    from spark_b200 import ops, step
    g = torch.Generator(device="cuda").manual_seed(6)
    n = 19
    gu = (torch.randn((n, 2 * i), generator=g, device="cuda") *
          torch.exp2(torch.randint(-14, 9, (n, 2 * i), generator=g, device="cuda").float())).to(torch.bfloat16)
    u = gu.view(torch.int16).cpu().numpy().view(np.uint16)
    silu = ops.act_mul_rows(gu).view(torch.int16).cpu().numpy().view(np.uint16)
    gelu = ops.act_mul_rows(gu, step.gelu_table("cuda")).view(torch.int16).cpu().numpy().view(np.uint16)
    table = oracle.gelu_table()
    for r in range(n):
        assert np.array_equal(silu[r], oracle.silu_mul(u[r, :i], u[r, i:])), r
        assert np.array_equal(gelu[r], oracle.gelu_mul(u[r, :i], u[r, i:], table)), r
