"""Tensor-parallel host logic on the CPU: the rank shards of every weight and the
claim the TP engine rests on -- a rank's o_proj / down_proj parts over its K shard
are exactly the single-GPU parts tp * kp .. of the whole matrix (checked through
the oracle's persistent-step GEMV), row shards give the same rows -- plus the part
counts at tp 2 / 4 / 8, the exchange-window layout and the handle exchange over a
world-size-2 gloo group."""
from __future__ import annotations

import os
import types

import numpy as np
import pytest
import torch


def _q4(n, k, seed, oracle):
    rng = np.random.default_rng(seed)
    qs, d = oracle.q4_quantize((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    return qs, d


def _full(cfg, oracle, seed=3):
    from spark_b200.model import LayerWeights, Q4Linear
    h, i, nq, D = cfg.hidden_size, cfg.intermediate_size, cfg.num_q_heads, cfg.head_dim

    def lin(n, k, s):
        qs, d = _q4(n, k, s, oracle)
        return Q4Linear(torch.from_numpy(qs), torch.from_numpy(d.view(np.int16)).view(torch.float16))

    layer = LayerWeights(in_norm=None, post_norm=None, qkv=lin(cfg.qkv_rows, h, seed), o=lin(h, nq * D, seed + 1),
                         gate_up=lin(2 * i, h, seed + 2), down=lin(h, i, seed + 3))
    return types.SimpleNamespace(cfg=cfg, device=torch.device("cpu"), layers=[layer], embed=None, final_norm=None,
                                 cos_sin=None, head=lin(cfg.vocab_size, h, seed + 4))


def _np(lin):
    return lin.qs.numpy(), lin.d.view(torch.int16).numpy().view(np.uint16)


def _x(k, seed):
    from oracle import f32_to_bf16
    return f32_to_bf16(np.random.default_rng(seed).standard_normal(k).astype(np.float32))


@pytest.mark.parametrize("tp", [2, 4])
def test_shards_reproduce_the_single_gpu_order(oracle, tp):
    from spark_b200 import step, tp as T
    from spark_b200.config import tiny_config
    cfg = tiny_config(num_layers=1, num_q_heads=8, num_kv_heads=4, vocab_size=512)
    full = _full(cfg, oracle)
    order = step.default_order(T.local_config(cfg, tp), 148, tp)
    kp_o, kp_d = order["kp_local"]
    assert order["kp"] == (tp * kp_o, tp * kp_d)
    ks = order["ks"]
    fl = full.layers[0]
    h, i = cfg.hidden_size, cfg.intermediate_size
    xo, xd, xh = _x(cfg.num_q_heads * cfg.head_dim, 1), _x(i, 2), _x(h, 3)
    o_full = oracle.t16_gemv_parts(xo, *_np(fl.o), tp * kp_o, ks[1])
    d_full = oracle.t16_gemv_parts(xd, *_np(fl.down), tp * kp_d, ks[3])
    qkv_full = oracle.t16_gemv(xh, *_np(fl.qkv), 1, ks[0])
    gu_full = oracle.t16_gemv(xh, *_np(fl.gate_up), 1, ks[2])
    head_full = oracle.t16_gemv(xh, *_np(full.head), 1, ks[4])
    ko, kd = xo.size // tp, i // tp
    for r in range(tp):
        sh = T.ShardWeights(full, r, tp)
        l = sh.layers[0]
        assert np.array_equal(oracle.t16_gemv_parts(xo[r * ko:(r + 1) * ko], *_np(l.o), kp_o, ks[1]),
                              o_full[r * kp_o:(r + 1) * kp_o])
        assert np.array_equal(oracle.t16_gemv_parts(xd[r * kd:(r + 1) * kd], *_np(l.down), kp_d, ks[3]),
                              d_full[r * kp_d:(r + 1) * kp_d])
        assert np.array_equal(oracle.t16_gemv(xh, *_np(l.qkv), 1, ks[0]), qkv_full[T.qkv_rows(cfg, r, tp).numpy()])
        assert np.array_equal(oracle.t16_gemv(xh, *_np(l.gate_up), 1, ks[2]),
                              gu_full[T.gate_up_rows(cfg, r, tp).numpy()])
        vl = cfg.vocab_size // tp
        assert sh.vocab_start == r * vl
        assert np.array_equal(oracle.t16_gemv(xh, *_np(sh.head), 1, ks[4]), head_full[r * vl:(r + 1) * vl])
    # the parts in rank order sum to the single-GPU bf16 result of the same order
    assert np.array_equal(oracle.parts_to_bf16(o_full),
                          oracle.t16_gemv(xo, *_np(fl.o), tp * kp_o, ks[1]))


def test_qkv_rows_are_head_aligned():
    from spark_b200 import tp as T
    from spark_b200.config import SparkConfig
    cfg = SparkConfig()
    rows = [T.qkv_rows(cfg, r, 2) for r in range(2)]
    allr = torch.cat(rows).sort().values
    assert torch.equal(allr, torch.arange(cfg.qkv_rows))
    D = cfg.head_dim
    assert rows[0][:D].tolist() == list(range(D))                      # q head 0
    assert rows[1][:D].tolist() == list(range(16 * D, 17 * D))         # q head 16
    assert rows[1][16 * D:17 * D].tolist() == list(range((32 + 4) * D, (32 + 5) * D))  # k head 4


@pytest.mark.parametrize("tp", [1, 2, 4, 8])
def test_full_model_part_counts(tp):
    from spark_b200 import step, tp as T
    from spark_b200.config import SparkConfig
    cfg = SparkConfig()
    loc = T.local_config(cfg, tp) if tp > 1 else cfg
    order = step.default_order(loc, 148, tp)
    kp_o, kp_d = order["kp_local"]
    assert tp * kp_o <= step.MAX_PARTS and tp * kp_d <= step.MAX_PARTS
    assert (loc.num_q_heads * loc.head_dim // kp_o) % 64 == 0
    assert (loc.intermediate_size // kp_d) % 64 == 0
    assert loc.vocab_size % 16 == 0 and loc.num_q_heads == 4 * loc.num_kv_heads
    if tp == 1:
        assert order["kp"] == (2, 4)


def test_tp_rejects_indivisible():
    from spark_b200 import tp as T
    from spark_b200.config import SparkConfig
    with pytest.raises(ValueError):
        T.local_config(SparkConfig(), 3)


def test_window_layout_aligned():
    from spark_b200 import tp as T
    from spark_b200.config import SparkConfig
    from spark_b200 import step
    cfg = T.local_config(SparkConfig(), 2)
    order = step.default_order(cfg, 148, 2, step.attn_splits(cfg, 148, 4096))
    fields = T.window_fields(cfg, order, T.program_stages(cfg.num_layers), 2)
    off, total = T.window_layout(fields)
    assert all(v % 256 == 0 for v in off.values())
    assert off["counters"] == 0 and total >= off["down_parts"] + 4 * 2 * order["kp_local"][1] * cfg.hidden_size
    # tagged exchange: per-layer words (8 bytes) of o_proj and down, every rank's parts
    off, total = T.window_layout(T.window_fields(cfg, order, T.program_stages(cfg.num_layers), 2, tagged=True))
    L, h = cfg.num_layers, cfg.hidden_size
    assert all(v % 256 == 0 for v in off.values()) and off["counters"] == 0
    assert off["down_tag"] >= off["o_tag"] + 8 * L * 2 * order["kp_local"][0] * h
    assert total >= off["down_tag"] + 8 * L * 2 * order["kp_local"][1] * h


def _gather_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from spark_b200 import tp as T
    got = T.gather_handles(bytes([rank + 1]) * T.IPC_HANDLE_BYTES, world)
    q.put((rank, [h[0] for h in got]))
    dist.destroy_process_group()


def test_handle_exchange_gloo_world2():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29000 + os.getpid() % 1000
    ps = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res == {0: [1, 2], 1: [1, 2]}
