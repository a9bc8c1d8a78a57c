"""One rank of the tensor-parallel decode parity run (launched by test_gpu_tp.py
through torch.distributed.run, one process per GPU).

Every rank builds the full synthetic weights from the same seed, keeps its shard
(spark_b200.tp.ShardWeights), decodes greedily with the persistent step kernel and
its in-kernel exchange, and checks that all ranks produced the same tokens.  Rank 0
then replays the same prompt through the CPU oracle in the order the ranks jointly
compute (tp x kp parts, the ranks' attention splits) and requires identical tokens
and bit-identical logits (the vocab shards gathered from all ranks).

    python -m torch.distributed.run --nproc-per-node 2 tests/tp_worker.py --new-tokens 64
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "spark-vllm-ascend_b200"))
sys.path.insert(0, ROOT)


def u16(t):
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", choices=["tiny", "full", "spark-tiny", "kv8"], default="tiny")
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--prompt", type=int, default=24)
    ap.add_argument("--new-tokens", type=int, default=64)
    ap.add_argument("--max-seq", type=int, default=256)
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--no-oracle", action="store_true")
    ap.add_argument("--exchange", choices=["counted", "tagged"], default="counted",
                    help="how o_proj / down parts cross the ranks (DecodeEngine tp_exchange)")
    ap.add_argument("--trace-ctx", type=int, default=0,
                    help="after the parity run: rewind to this context, time 20 steps, then trace one step "
                         "(per-stage timeline of rank 0, as spark_b200.step_trace prints it)")
    args = ap.parse_args(argv)

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    from spark_b200 import tp as T
    from spark_b200.config import SparkConfig, spark_x26_config, tiny_config
    from spark_b200.model import DecodeEngine, SyntheticWeights

    kw = {"num_layers": args.layers} if args.layers else {}
    if args.config == "spark-tiny":  # the Spark architecture (gate, GELU, sliding window, Q6_K head)
        cfg = spark_x26_config(num_layers=args.layers or 4, hidden_size=512, num_q_heads=8, num_kv_heads=2,
                               intermediate_size=1024, vocab_size=4096, sliding_window=33, max_position=4096,
                               name="spark-tiny")
    elif args.config == "kv8":  # the 4B model's head layout (32 q / 8 kv heads of 128) at a small size:
        # shards over 2, 4 and 8 ranks (intermediate 1024 / 8 = 128 rows, vocab 4096 / 8 per rank)
        cfg = tiny_config(hidden_size=512, num_q_heads=32, num_kv_heads=8, intermediate_size=1024,
                          vocab_size=4096, name="spark-kv8", **kw)
    else:
        cfg = tiny_config(**kw) if args.config == "tiny" else SparkConfig(max_position=4096, **kw)
    full = SyntheticWeights(cfg, device="cuda", seed=args.seed)
    shard = T.ShardWeights(full, rank, world)
    host_weights = full.to_numpy() if rank == 0 and not args.no_oracle else None
    del full
    eng = DecodeEngine(shard, max_seq_len=args.max_seq, num_blocks=4 * ((args.max_seq + 127) // 128),
                       seed=args.seed, mode="step", tp_exchange=args.exchange)
    rng = np.random.default_rng(args.seed)
    prompt = rng.integers(0, cfg.vocab_size, args.prompt).astype(np.int32)
    toks = eng.generate(torch.from_numpy(prompt), args.new_tokens)
    torch.cuda.synchronize()
    err = int(eng.error.item())
    logits = torch.from_numpy(u16(eng.logits).astype(np.int32)).cuda()
    all_logits = [torch.empty_like(logits) for _ in range(world)]
    dist.all_gather(all_logits, logits)
    all_toks: list = [None] * world
    dist.all_gather_object(all_toks, toks)
    res = {"rank": rank, "world": world, "error": err, "splits": eng.splits, "order": eng.oracle_order(),
           "ranks_agree": all(t == toks for t in all_toks), "tokens": toks[:8]}
    ok = err == 0 and res["ranks_agree"]
    if rank == 0 and not args.no_oracle:
        import oracle
        if cfg.spark_features:
            om = oracle.SparkOracleModel(cfg, host_weights, eng.num_blocks, eng.splits, eng.oracle_order())
        else:
            om = oracle.OracleModel(cfg, host_weights, num_blocks=eng.num_blocks, splits=eng.splits,
                                    order=eng.oracle_order())
        table = eng.block_table.cpu().numpy()
        pos, tok = 0, None
        for t in prompt:
            tok = om.step(table, int(t), pos)
            pos += 1
        ref, ref_logits = [tok], None
        for i in range(args.new_tokens - 1):
            want = i == args.new_tokens - 2
            r = om.step(table, ref[-1], pos, want_logits=want)
            if want:
                r, ref_logits = r
            ref.append(r)
            pos += 1
        got_logits = torch.cat(all_logits).cpu().numpy().astype(np.uint16)
        res["oracle_tokens_equal"] = ref == toks
        res["oracle_logits_equal"] = bool(ref_logits is not None and np.array_equal(got_logits, ref_logits))
        ok = ok and res["oracle_tokens_equal"] and res["oracle_logits_equal"]
    res["ok"] = ok
    print(json.dumps(res), flush=True)
    if args.trace_ctx:
        from spark_b200.step_trace import stage_kinds, summarize
        eng.reset(args.trace_ctx)
        eng.token.fill_(1)
        for _ in range(4):
            eng.step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(20):
            eng.step()
        e1.record()
        torch.cuda.synchronize()
        tr = eng.program.trace_buffer()
        dist.barrier()
        eng.program.launch(eng.program.io(error=eng.error, key=eng.key, token_out=eng.token,
                                          token_log=eng.token_log, step=eng.step_idx, pos=eng.pos,
                                          window=eng.window, trace=tr))
        torch.cuda.synchronize()
        t = tr.cpu().numpy().astype(np.int64)
        if rank == 0:
            print(json.dumps({"trace_ctx": args.trace_ctx, "ms_per_step": round(e0.elapsed_time(e1) / 20, 4),
                              "stages": summarize(t, stage_kinds(cfg.num_layers))}), flush=True)
    eng.close()
    dist.barrier()
    dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
