"""End-to-end GPU parity of the decode engine against the CPU oracle model.

* Identical greedy tokens for the first 64 decode steps (north-star criterion),
  plus bit-identical logits after the last step, on a small synthetic model.
* The full-size synthetic 4B model (36 layers, vocab 151936): a few prefill and
  decode steps with the same check, so every real shape goes through the graph.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def u16(t):
    import torch
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _run_pair(cfg, prompt_len, new_tokens, splits, max_seq, seed, oracle, use_graph=True, mode="step"):
    import torch
    from spark_b200.model import DecodeEngine, SyntheticWeights
    w = SyntheticWeights(cfg, device="cuda", seed=seed)
    eng = DecodeEngine(w, max_seq_len=max_seq, splits=splits if mode == "kernels" else 0,
                       num_blocks=4 * ((max_seq + 127) // 128), use_graph=use_graph, seed=seed, mode=mode)
    splits = eng.splits
    rng = np.random.default_rng(seed)
    prompt = rng.integers(0, cfg.vocab_size, prompt_len).astype(np.int32)
    toks = eng.generate(torch.from_numpy(prompt), new_tokens)
    torch.cuda.synchronize()
    assert int(eng.error.item()) == 0
    # oracle: same weights, same block table, same token-by-token feeding
    om = oracle.OracleModel(cfg, w.to_numpy(), num_blocks=eng.num_blocks, splits=splits, order=eng.oracle_order())
    table = eng.block_table.cpu().numpy()
    pos = 0
    tok = None
    for t in prompt:
        tok = om.step(table, int(t), pos)
        pos += 1
    ref = [tok]
    logits = None
    for i in range(new_tokens - 1):
        want = i == new_tokens - 2
        r = om.step(table, ref[-1], pos, want_logits=want)
        if want:
            r, logits = r
        ref.append(r)
        pos += 1
    return toks, ref, u16(eng.logits), logits, eng


@pytest.mark.parametrize("mode", ["step", "kernels"])
def test_tiny_model_greedy_64_steps(cuda, oracle, mode):
    from spark_b200.config import tiny_config
    cfg = tiny_config()
    toks, ref, lg, ref_lg, eng = _run_pair(cfg, prompt_len=24, new_tokens=65, splits=4, max_seq=256, seed=1,
                                           oracle=oracle, mode=mode)
    assert toks == ref
    assert np.array_equal(lg, ref_lg)
    assert eng.kernels_per_step() == (1 if mode == "step" else 5 * cfg.num_layers + 2)


@pytest.mark.parametrize("mode", ["step", "kernels"])
def test_tiny_model_eager_matches_graph(cuda, oracle, mode):
    from spark_b200.config import tiny_config
    cfg = tiny_config(num_layers=3)
    toks, ref, _, _, _ = _run_pair(cfg, prompt_len=5, new_tokens=9, splits=2, max_seq=128, seed=2, oracle=oracle,
                                   use_graph=False, mode=mode)
    assert toks == ref


@pytest.mark.slow
@pytest.mark.parametrize("mode", ["step", "kernels"])
def test_full_size_model_steps(cuda, oracle, mode):
    from spark_b200.config import SparkConfig
    cfg = SparkConfig(max_position=4096)
    toks, ref, lg, ref_lg, _ = _run_pair(cfg, prompt_len=3, new_tokens=3, splits=16, max_seq=512, seed=3,
                                         oracle=oracle, mode=mode)
    assert toks == ref
    assert np.array_equal(lg, ref_lg)


def test_long_context_decode_matches_oracle(cuda, oracle):
    """Context 32000+ on the persistent step: 37 splits per kv head (296 (kv head, split)
    tasks on 148 CTAs, two in turn on each); a random KV cache, two decode steps,
    identical tokens and logits to the oracle.  Two layers keep the caches small."""
    import torch
    from spark_b200.config import SparkConfig
    from spark_b200.model import DecodeEngine, SyntheticWeights
    cfg = SparkConfig(num_layers=2)
    w = SyntheticWeights(cfg, device="cuda", seed=5)
    max_seq = 32768
    eng = DecodeEngine(w, max_seq_len=max_seq, num_blocks=max_seq // 128 + 4, seed=5, mode="step")
    assert eng.splits * cfg.num_kv_heads > eng.ncta
    g = torch.Generator(device="cuda").manual_seed(5)
    eng.k_cache.copy_(torch.randn(eng.k_cache.shape, generator=g, device="cuda").to(torch.bfloat16))
    eng.v_cache.copy_(torch.randn(eng.v_cache.shape, generator=g, device="cuda").to(torch.bfloat16))
    pos0 = 32000
    om = oracle.OracleModel(cfg, w.to_numpy(), num_blocks=eng.num_blocks, splits=eng.splits,
                            order=eng.oracle_order())
    om.kc[...] = u16(eng.k_cache).reshape(om.kc.shape)
    om.vc[...] = u16(eng.v_cache).reshape(om.vc.shape)
    eng.reset(pos0)
    eng.set_token(123)
    table = eng.block_table.cpu().numpy()
    tok = 123
    for i in range(2):
        eng.step()
        torch.cuda.synchronize()
        want, want_lg = om.step(table, tok, pos0 + i, want_logits=True)
        assert int(eng.error.item()) == 0
        assert int(eng.token.item()) == want
        assert np.array_equal(u16(eng.logits), want_lg)
        tok = want



@pytest.mark.slow
def test_full_model_2048_prompt_greedy_64_tokens(cuda, oracle):
    """The north-star parity criterion on the benchmark model itself:
    the 36-layer synthetic 4B Q4_0 model, a seeded 2048-token prompt through the batched
    GPU prefill, then 64 greedy decode steps of the persistent step kernel.  The CPU oracle
    decodes from the same KV cache (the prefill's output) and must produce identical
    tokens and, after the last step, bit-identical logits."""
    import torch
    from spark_b200.config import SparkConfig
    from spark_b200.model import DecodeEngine, SyntheticWeights
    cfg = SparkConfig()
    w = SyntheticWeights(cfg, device="cuda", seed=21)
    P, N = 2048, 64
    max_seq = P + N + 1
    eng = DecodeEngine(w, max_seq_len=max_seq, num_blocks=(max_seq + 127) // 128 + 4, seed=21, mode="step")
    prompt = np.random.default_rng(21).integers(0, cfg.vocab_size, P).astype(np.int32)
    first = int(eng.prefill_batched(torch.from_numpy(prompt)).item())
    torch.cuda.synchronize()
    om = oracle.OracleModel(cfg, w.to_numpy(), num_blocks=eng.num_blocks, splits=eng.splits,
                            order=eng.oracle_order())
    om.kc[...] = u16(eng.k_cache).reshape(om.kc.shape)
    om.vc[...] = u16(eng.v_cache).reshape(om.vc.shape)
    table = eng.block_table.cpu().numpy()
    eng.step_idx.zero_()
    for _ in range(N):
        eng.step()
    torch.cuda.synchronize()
    assert int(eng.error.item()) == 0
    gpu = eng.token_log[:N].cpu().tolist()
    gpu_lg = u16(eng.logits)
    tok, ref, ref_lg = first, [], None
    for i in range(N):
        r = om.step(table, tok, P + i, want_logits=i == N - 1)
        if i == N - 1:
            r, ref_lg = r
        ref.append(int(r))
        tok = int(r)
    assert gpu == ref
    assert np.array_equal(gpu_lg, ref_lg)
