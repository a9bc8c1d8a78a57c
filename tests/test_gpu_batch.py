"""Small-batch decode (BASELINE configs[4]'s batch 2 / 4 / 8): B sequences through one
persistent launch per step.  Every sequence must decode exactly as the CPU oracle decodes
it alone (the one-sequence order of the batch program, ``BatchDecodeEngine.oracle_order``):
identical tokens every step and bit-identical logits.  The sequences sit at different
positions over one shared paged cache (disjoint blocks per sequence), filled with random
K / V so that long contexts need no prefill."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def u16(t):
    import torch
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _run(cuda, oracle, cfg, batch, positions, steps, seed, max_seq):
    import torch
    from spark_b200.batch import BatchDecodeEngine
    from spark_b200.model import SyntheticWeights
    w = SyntheticWeights(cfg, device="cuda", seed=seed)
    eng = BatchDecodeEngine(w, batch, max_seq_len=max_seq, seed=seed)
    g = torch.Generator(device="cuda").manual_seed(seed)
    eng.k_cache.copy_(torch.randn(eng.k_cache.shape, generator=g, device="cuda").to(torch.bfloat16))
    eng.v_cache.copy_(torch.randn(eng.v_cache.shape, generator=g, device="cuda").to(torch.bfloat16))
    om = oracle.OracleModel(cfg, w.to_numpy(), num_blocks=eng.num_blocks, splits=eng.splits,
                            order=eng.oracle_order())
    om.kc[...] = u16(eng.k_cache).reshape(om.kc.shape)
    om.vc[...] = u16(eng.v_cache).reshape(om.vc.shape)
    tables = eng.block_tables.cpu().numpy()
    toks = np.random.default_rng(seed).integers(0, cfg.vocab_size, batch).tolist()
    eng.reset_counters()
    eng.set_positions(positions)
    eng.token.copy_(torch.tensor(toks, dtype=torch.int32))
    for i in range(steps):
        eng.step()
        torch.cuda.synchronize()
        assert int(eng.error.item()) == 0
        got = eng.token.cpu().tolist()
        last = i == steps - 1
        for b in range(batch):
            r = om.step(tables[b], toks[b], positions[b] + i, want_logits=last)
            if last:
                r, lg = r
                assert np.array_equal(u16(eng.logits[b]), lg), (b, i)
            assert got[b] == int(r), (b, i, got[b], int(r))
        toks = got
    assert eng.pos.cpu().tolist() == [p + steps for p in positions]
    return eng


@pytest.mark.parametrize("batch", [2, 4, 8])
def test_batch_tiny_matches_oracle(cuda, oracle, batch):
    """Tiny model, 3 layers, sequences at positions 60 + 37 b: 12 steps."""
    from spark_b200.config import tiny_config
    cfg = tiny_config(num_layers=3)
    positions = [60 + 37 * b for b in range(batch)]
    _run(cuda, oracle, cfg, batch, positions, steps=12, seed=31 + batch, max_seq=512)


@pytest.mark.parametrize("batch", [2, 4, 8])
def test_batch_4b_long_context_matches_oracle(cuda, oracle, batch):
    """The 4B shapes (hidden 2560, 32 q / 8 kv heads, SwiGLU 9728, vocab 151936; two
    layers keep the caches small) at configs[4]'s context: sequences near position 32K
    (b-th at 32000 - 700 b), several (sequence, kv head, split) tasks per CTA; 2 steps."""
    from spark_b200.config import SparkConfig
    cfg = SparkConfig(num_layers=2)
    positions = [32000 - 700 * b for b in range(batch)]
    eng = _run(cuda, oracle, cfg, batch, positions, steps=2, seed=41 + batch, max_seq=32768)
    assert batch * cfg.num_kv_heads * eng.splits > eng.ncta


def test_batch_generate_matches_oracle_tokens(cuda, oracle):
    """Prompts of one length fed through the batch decode path (stepwise prefill), then
    greedy tokens: each sequence identical to the oracle's token-by-token decode."""
    import torch
    from spark_b200.batch import BatchDecodeEngine
    from spark_b200.config import tiny_config
    from spark_b200.model import SyntheticWeights
    cfg = tiny_config()
    B, P, N = 4, 10, 20
    w = SyntheticWeights(cfg, device="cuda", seed=51)
    eng = BatchDecodeEngine(w, B, max_seq_len=64, seed=51)
    prompts = np.random.default_rng(51).integers(0, cfg.vocab_size, (B, P)).tolist()
    out = eng.generate(prompts, N, stepwise=True)
    assert int(eng.error.item()) == 0
    om = oracle.OracleModel(cfg, w.to_numpy(), num_blocks=eng.num_blocks, splits=eng.splits,
                            order=eng.oracle_order())
    tables = eng.block_tables.cpu().numpy()
    for b in range(B):
        tok = None
        for i, t in enumerate(prompts[b]):
            tok = om.step(tables[b], int(t), i)
        ref = [int(tok)]
        for i in range(N - 1):
            ref.append(int(om.step(tables[b], ref[-1], P + i)))
        assert out[b] == ref, b


def test_batch_program_rejects_unsupported_forms(cuda):
    """The host refuses what the batch kernels do not carry: a batch of 3, mixed batches,
    4-slice units."""
    import torch
    from spark_b200 import step as S
    from spark_b200._lib import SparkError
    with pytest.raises(ValueError):
        S.StepProgram("cuda", batch=3)
    x = torch.zeros((2, 256), dtype=torch.bfloat16, device="cuda")
    wq = torch.zeros(S.t16_bytes(64, 256, 1), dtype=torch.uint8, device="cuda")
    out = torch.zeros((2, 64), dtype=torch.bfloat16, device="cuda")
    prog = S.StepProgram("cuda", batch=2)
    prog.gemv(wq, 64, 256, ks=4, a=x, out=out)
    prog.finalize()
    with pytest.raises(SparkError):
        prog.launch(prog.io())
