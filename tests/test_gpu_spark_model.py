"""End-to-end GPU parity of the Spark architecture (the reference's served model,
plugin/spark2_5.py): headwise output gate, GELU * mul, sliding-window and
partial-RoPE full layers, head_dim 256, tied Q6_K embedding as LM head -- all in one
persistent-step launch per token, token- and logit-identical to the oracle's
SparkOracleModel.

* a small Spark-shaped model over a prompt longer than its sliding window, then
  greedy decode;
* the Spark-X2.6-4B layer shapes (hidden 2560, 16 q / 4 kv heads of 256, intermediate
  10240, vocab 131072 Q6_K head) with one sliding and one full layer, decoding past
  the window over a random KV cache.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def u16(t):
    import torch
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def test_tiny_spark_model_greedy(cuda, oracle):
    import torch
    from spark_b200.config import spark_x26_config
    from spark_b200.model import DecodeEngine, SyntheticWeights
    cfg = spark_x26_config(num_layers=4, hidden_size=512, num_q_heads=8, num_kv_heads=2, intermediate_size=1024,
                           vocab_size=4096, sliding_window=33, max_position=4096, name="spark-tiny")
    assert cfg.layer_types == ("sliding_attention",) * 3 + ("full_attention",)
    w = SyntheticWeights(cfg, device="cuda", seed=4)
    eng = DecodeEngine(w, max_seq_len=256, num_blocks=8, seed=4)
    rng = np.random.default_rng(4)
    prompt = rng.integers(0, cfg.vocab_size, 70).astype(np.int32)
    new = 24
    toks = eng.generate(torch.from_numpy(prompt), new)
    torch.cuda.synchronize()
    assert int(eng.error.item()) == 0
    om = oracle.SparkOracleModel(cfg, w.to_numpy(), eng.num_blocks, eng.splits, eng.oracle_order())
    table = eng.block_table.cpu().numpy()
    tok = None
    for pos, t in enumerate(prompt):
        tok = om.step(table, int(t), pos)
    ref = [tok]
    logits = None
    for i in range(new - 1):
        r, logits = om.step(table, ref[-1], len(prompt) + i, want_logits=True)
        ref.append(r)
    assert toks == ref
    assert np.array_equal(u16(eng.logits), logits)


def test_spark_x26_shapes_decode(cuda, oracle):
    import torch
    from spark_b200.config import spark_x26_config
    from spark_b200.model import DecodeEngine, SyntheticWeights
    cfg = spark_x26_config(num_layers=2, layer_types=("sliding_attention", "full_attention"), max_position=8192)
    w = SyntheticWeights(cfg, device="cuda", seed=6)
    max_seq = 4096
    eng = DecodeEngine(w, max_seq_len=max_seq, num_blocks=max_seq // 128 + 4, seed=6)
    g = torch.Generator(device="cuda").manual_seed(6)
    eng.k_cache.copy_(torch.randn(eng.k_cache.shape, generator=g, device="cuda").to(torch.bfloat16))
    eng.v_cache.copy_(torch.randn(eng.v_cache.shape, generator=g, device="cuda").to(torch.bfloat16))
    om = oracle.SparkOracleModel(cfg, w.to_numpy(), eng.num_blocks, eng.splits, eng.oracle_order())
    om.kc[...] = u16(eng.k_cache).reshape(om.kc.shape)
    om.vc[...] = u16(eng.v_cache).reshape(om.vc.shape)
    pos0 = 3001
    eng.reset(pos0)
    eng.set_token(77)
    table = eng.block_table.cpu().numpy()
    tok = 77
    for i in range(3):
        eng.step()
        torch.cuda.synchronize()
        want, want_lg = om.step(table, tok, pos0 + i, want_logits=True)
        assert int(eng.error.item()) == 0
        assert np.array_equal(u16(eng.logits), want_lg)
        assert int(eng.token.item()) == want
        tok = want
