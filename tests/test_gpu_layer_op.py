"""The reference's per-layer op contract, ``torch.ops.spark_b200.layer_run(x, residual,
positions, key) -> (x, residual)`` (reference integration/model.py:46-82, called per layer
by plugin/spark2_5.py:369-376), run the way the reference's model forward runs it: the
first input norm, then layer_run over every layer, then greedy argmax over the LM head of
the final normalized state.  Checked against the CPU oracle composed from the same
primitives in the op's order, bit for bit (normalized state, residual, K / V cache
contents, tokens)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def u16(t):
    import torch
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _oracle_layer(oracle, cfg, w, li, x, res, pos, kc, vc, table, splits, order, down_ks, next_norm):
    nq, nkv, D, bs, I = cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim, cfg.block_size, cfg.intermediate_size
    p = f"layers.{li}."
    ks_qkv, ks_o, ks_gu, _, _ = order["ks"]
    kp_o = order["kp_local"][0]
    qkv = oracle.t16_gemv(x, w[p + "qkv_qs"], w[p + "qkv_d"], 1, ks_qkv).reshape(nq + 2 * nkv, D)
    qk = oracle.rope_neox(qkv[:nq + nkv], w["cos_sin"][pos])
    blk = table[pos // bs]
    kc[blk, :, pos % bs] = qk[nq:]
    vc[blk, :, pos % bs] = qkv[nq + nkv:]
    po, pl = oracle.attn_split(qk[:nq], kc, vc, table, pos + 1, splits, cfg.attn_scale, chunk_accs=11)
    attn = oracle.attn_combine(po, pl).reshape(-1)
    a_o = oracle.parts_to_bf16(oracle.t16_gemv_parts(attn, w[p + "o_qs"], w[p + "o_d"], kp_o, ks_o))
    res1, x2 = oracle.add_rmsnorm(a_o, res, w[p + "post_norm"], cfg.rms_norm_eps)
    gu = oracle.t16_gemv(x2, w[p + "gu_qs"], w[p + "gu_d"], 1, ks_gu)
    mid = oracle.silu_mul(gu[:I], gu[I:])
    a_d = oracle.t16_gemv(mid, w[p + "down_qs"], w[p + "down_d"], 1, down_ks)
    res2, y = oracle.add_rmsnorm(a_d, res1, next_norm, cfg.rms_norm_eps)
    return y, res2


def test_layer_run_matches_oracle(cuda, oracle):
    import torch
    from spark_b200 import layer_op, ops
    from spark_b200.config import tiny_config
    from spark_b200.model import SyntheticWeights
    cfg = tiny_config(num_layers=3)
    w = SyntheticWeights(cfg, device="cuda", seed=7)
    wn = w.to_numpy()
    L, nkv, bs, D = cfg.num_layers, cfg.num_kv_heads, cfg.block_size, cfg.head_dim
    max_seq, nblk = 256, 8
    table = torch.randperm(nblk, generator=torch.Generator().manual_seed(7))[: max_seq // bs].to(torch.int32)
    table_d = table.to(cuda)
    kc = torch.zeros((L, nblk, nkv, bs, D), dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    layer_op.unregister_all()
    binds = []
    for li, lw in enumerate(w.layers):
        nxt = w.layers[li + 1].in_norm if li + 1 < L else w.final_norm
        b = layer_op.LayerBinding(cfg, lw, nxt, w.cos_sin, kc[li], vc[li], table_d, max_seq)
        layer_op.register_layer(f"model.layers.{li}.self_attn", b)
        binds.append(b)
    okc = np.zeros((L, nblk, nkv, bs, D), np.uint16)
    ovc = np.zeros_like(okc)
    tnp = table.numpy()
    rng = np.random.default_rng(7)
    tokens = rng.integers(0, cfg.vocab_size, 6).tolist()
    gen = []
    for pos in range(20):
        tok = tokens[pos] if pos < len(tokens) else gen[-1]
        emb = w.embed[tok]
        x, res = torch.ops.spark_b200.add_rmsnorm(emb, None, w.layers[0].in_norm, cfg.rms_norm_eps)
        ores, ox = oracle.add_rmsnorm(wn["embed"][tok], None, wn["layers.0.in_norm"], cfg.rms_norm_eps)
        positions = torch.tensor([pos], dtype=torch.int64, device=cuda)
        x, res = x.reshape(1, -1), res.reshape(1, -1)
        for li in range(L):
            x, res = torch.ops.spark_b200.layer_run(x, res, positions, f"model.layers.{li}.self_attn")
            nxt = wn[f"layers.{li + 1}.in_norm"] if li + 1 < L else wn["final_norm"]
            ox, ores = _oracle_layer(oracle, cfg, wn, li, ox, ores, pos, okc[li], ovc[li], tnp,
                                     binds[li].splits, binds[li].order, binds[li].order_down[1], nxt)
            torch.cuda.synchronize()
            assert np.array_equal(u16(x).reshape(-1), ox), (pos, li)
            assert np.array_equal(u16(res).reshape(-1), ores), (pos, li)
        logits = ops.q4_gemv(x, w.head.qs, w.head.d)
        nxt_tok = int(torch.argmax(logits.float().reshape(-1)).item())
        if pos >= len(tokens) - 1:
            gen.append(nxt_tok)
    assert all(int(b.error.item()) == 0 for b in binds)
    assert np.array_equal(u16(kc), okc) and np.array_equal(u16(vc), ovc)
    assert len(gen) == 20 - len(tokens) + 1
