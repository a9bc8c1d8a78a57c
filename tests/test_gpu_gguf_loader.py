"""GPU round trip of the GGUF loader: a Spark-architecture model written as a GGUF with
the reference checkpoint's tensor names (tests/gguf_fixture.py) loads back into
bit-identical engine weights (Q4_0 planes split on the device, F32 norms, the tied
Q6_K embedding and its bf16 decode), and the engine built from the file decodes the
same greedy tokens and logits as the engine built from the source weights."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_gguf_round_trip_and_decode(cuda, oracle, tmp_path):
    import torch
    from gguf_fixture import write_spark_gguf
    from spark_b200.config import spark_x26_config
    from spark_b200.gguf_loader import load_gguf
    from spark_b200.model import DecodeEngine, SyntheticWeights
    cfg = spark_x26_config(num_layers=4, hidden_size=512, num_q_heads=8, num_kv_heads=2, intermediate_size=1024,
                           vocab_size=4096, sliding_window=33, max_position=4096, name="spark-tiny")
    src = SyntheticWeights(cfg, device="cuda", seed=9)
    ref = src.to_numpy()
    path = write_spark_gguf(tmp_path / "spark.gguf", cfg, ref, oracle)
    got = load_gguf(path, cfg).to_numpy()
    assert sorted(got) == sorted(ref)
    for k in ref:
        assert np.array_equal(got[k], ref[k]), k
    toks = []
    for w in (src, load_gguf(path, cfg)):
        eng = DecodeEngine(w, max_seq_len=128, num_blocks=4, seed=9)
        toks.append((eng.generate(torch.arange(20, dtype=torch.int32) * 37 % cfg.vocab_size, 12),
                     eng.logits.clone()))
    assert toks[0][0] == toks[1][0]
    assert torch.equal(toks[0][1], toks[1][1])


def test_gguf_separate_qkv_untied_head(cuda, oracle, tmp_path):
    """The llama-style layout the loader also reads: separate attn_q / attn_k / attn_v,
    a float token_embd and a Q4_0 output head (the synthetic 4B architecture, small)."""
    import torch
    from gguf_fixture import write_spark_gguf
    from spark_b200.config import tiny_config
    from spark_b200.gguf_loader import load_gguf
    from spark_b200.model import DecodeEngine, SyntheticWeights
    cfg = tiny_config(num_layers=2)
    src = SyntheticWeights(cfg, device="cuda", seed=10)
    ref = src.to_numpy()
    path = write_spark_gguf(tmp_path / "llama.gguf", cfg, ref, oracle, fused_qkv=False)
    got = load_gguf(path, cfg).to_numpy()
    assert sorted(got) == sorted(ref)
    for k in ref:
        assert np.array_equal(got[k], ref[k]), k
    toks = [DecodeEngine(w, max_seq_len=128, num_blocks=4, seed=10).generate(
        torch.arange(9, dtype=torch.int32) * 53 % cfg.vocab_size, 6) for w in (src, load_gguf(path, cfg))]
    assert toks[0] == toks[1]
