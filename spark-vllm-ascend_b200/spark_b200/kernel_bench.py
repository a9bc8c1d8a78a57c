"""Per-kernel HBM bandwidth of the decode hot path (BASELINE configs[0] and [1]).

    python -m spark_b200.kernel_bench [--kernels gemv,gate_up,...] [--reps N] [--copies C]

Every kernel is timed with CUDA events over ``reps`` back-to-back launches that
rotate through ``copies`` independent weight / KV sets (more bytes than the 126 MB
L2), so each launch reads its operands from HBM.  Algorithmic bytes per launch are
the packed weights (18 B per 32 weights) plus activations in and out (GEMV), or the
K/V rows of the context plus q / out (attention).  Prints one JSON line.

Shapes (synthetic 4B model): qkv 6144x2560 (+RMSNorm, RoPE, KV store), o 2560x4096,
gate_up 19456x2560 (+RMSNorm, SiLU*mul), down 2560x9728, head 151936x2560 (+argmax),
and the single-op GEMV of configs[0]: 9728x2560.  Attention: 32 q / 8 kv heads,
head_dim 128, block 128, ctx {2048, 4096, 6144}, 16 splits.
"""
from __future__ import annotations

import argparse
import json
import math

import torch

from . import ops
from .config import SparkConfig
from .model import rope_cos_sin

BF16 = torch.bfloat16


def _q4(n, k, device, gen):
    w = torch.randn((n, k), generator=gen, device=device) * 0.02
    return ops.q4_quantize(w)


def _time(fn, reps):
    """Average device time of one launch: ``reps`` launches captured in a CUDA graph
    (no host launch overhead; consecutive launches overlap through PDL exactly as in
    the decode step), replayed after a warm-up replay."""
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for i in range(3):
            fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(reps):
            fn(i)
    with torch.cuda.stream(stream):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record()
        g.replay()
        e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps * 1e3  # us


def gemv_cases(cfg: SparkConfig):
    h, i = cfg.hidden_size, cfg.intermediate_size
    return {
        "gemv": (9728, h, "plain"),
        "qkv": (cfg.qkv_rows, h, "qkv"),
        "o_proj": (h, cfg.num_q_heads * cfg.head_dim, "plain"),
        "gate_up": (2 * i, h, "gate_up"),
        "down": (h, i, "plain"),
        "head": (cfg.vocab_size, h, "head"),
    }


def bench_gemv(name, n, k, kind, reps, copies, device, gen, cfg):
    wb = n * k // 32 * 18
    copies = max(1, min(copies, math.ceil(400e6 / wb)))
    ws = [_q4(n, k, device, gen) for _ in range(copies)]
    x = torch.randn(k, device=device).to(BF16)
    b = torch.randn(k, device=device).to(BF16)
    g = torch.ones(k, device=device, dtype=BF16)
    res = torch.empty(k, device=device, dtype=BF16)
    if kind == "plain":
        y = torch.empty(n, device=device, dtype=BF16)
        fn = lambda t: ops.q4_gemv_out(x, ws[t % copies][0], ws[t % copies][1], y)  # noqa: E731
        io = 2 * k + 2 * n
    elif kind == "gate_up":
        mid = torch.empty(n // 2, device=device, dtype=BF16)
        fn = lambda t: ops.rmsnorm_gate_up_silu_out(x, b, g, 1e-6, ws[t % copies][0], ws[t % copies][1], mid,  # noqa
                                                     res)
        io = 3 * 2 * k + n
    elif kind == "head":
        logits = torch.empty(n, device=device, dtype=BF16)
        key = torch.zeros(1, device=device, dtype=torch.int64)
        fn = lambda t: ops.head_argmax_out(x, b, g, 1e-6, ws[t % copies][0], ws[t % copies][1], logits, key)  # noqa
        io = 2 * 2 * k + 2 * n
    else:  # qkv
        D, nq, nkv = cfg.head_dim, cfg.num_q_heads, cfg.num_kv_heads
        cs = rope_cos_sin(cfg, 8192).to(device)
        kc = torch.zeros((64, nkv, cfg.block_size, D), device=device, dtype=BF16)
        vc = torch.zeros_like(kc)
        q = torch.empty((nq, D), device=device, dtype=BF16)
        pos = torch.tensor([1000], device=device, dtype=torch.int64)
        table = torch.arange(64, device=device, dtype=torch.int32)
        fn = lambda t: ops.qkv_rope_kvstore_out(x, b, g, 1e-6, ws[t % copies][0], ws[t % copies][1], nq, nkv, D, cs,  # noqa
                                                pos, table, None, cfg.block_size, kc, vc, q, res)
        io = 3 * 2 * k + 2 * n
    us = _time(fn, reps)
    byts = wb + io
    return {"us": round(us, 3), "bytes": byts, "gbs": round(byts / us / 1e3, 1), "copies": copies}


def bench_attn(ctx, splits, reps, copies, device, gen, cfg):
    nq, nkv, D, bs = cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim, cfg.block_size
    nblk = (ctx + bs - 1) // bs
    per = 2 * nblk * nkv * bs * D * 2
    copies = max(1, min(copies, math.ceil(400e6 / per)))
    caches = []
    for _ in range(copies):
        kc = torch.randn((nblk, nkv, bs, D), generator=gen, device=device).to(BF16)
        vc = torch.randn((nblk, nkv, bs, D), generator=gen, device=device).to(BF16)
        table = torch.randperm(nblk, device=device, generator=gen).to(torch.int32)
        caches.append((kc, vc, table))
    q = torch.randn((nq, D), device=device).to(BF16)
    pos = torch.tensor([ctx - 1], device=device, dtype=torch.int64)
    T = ((ctx + splits - 1) // splits + 15) // 16 * 16
    po = torch.empty((splits, nq, D), device=device, dtype=torch.float32)
    pl = torch.empty((splits, nq), device=device, dtype=torch.float32)
    out = torch.empty((nq, D), device=device, dtype=BF16)
    scale = cfg.attn_scale

    def split(t):
        kc, vc, table = caches[t % copies]
        ops.attn_splitkv_out(q, kc, vc, table, splits, T, scale, po, pl, pos=pos)

    def both(t):
        split(t)
        ops.attn_combine_out(po, pl, out)

    counters = torch.zeros(nkv, device=device, dtype=torch.int32)

    def fused(t):  # one launch: the last split of each kv head merges its heads
        kc, vc, table = caches[t % copies]
        ops.attn_decode_out(q, kc, vc, table, splits, T, scale, po, pl, counters, out, pos=pos)

    us_split = _time(split, reps)
    us_both = _time(both, reps)
    us_fused = _time(fused, reps)
    byts = 2 * ctx * nkv * D * 2 + 2 * nq * D * 2
    return {"us_split": round(us_split, 3), "us_split_combine": round(us_both, 3), "us_fused": round(us_fused, 3),
            "bytes": byts, "gbs_split": round(byts / us_split / 1e3, 1),
            "gbs_split_combine": round(byts / us_both / 1e3, 1), "gbs_fused": round(byts / us_fused / 1e3, 1)}


# ---------------------------------------------------------------- persistent-step stages
def bench_step_gemv(name, n, k, kind, reps, copies, device, gen, cfg):
    """One GEMV stage of the persistent decode-step kernel as its own launch (T16
    weights, the decode program's slice / part counts)."""
    from . import step as S
    order = S.default_order(cfg, S.num_ctas())
    ks_qkv, ks_o, ks_gu, ks_down, ks_head = order["ks"]
    kp_o, kp_down = order["kp"]
    spec = {"gemv": (1, ks_head, S.ROWS_PLAIN, S.EPI_BF16), "qkv": (1, ks_qkv, S.ROWS_PAIR_HALF, S.EPI_BF16),
            "o_proj": (kp_o, ks_o, S.ROWS_PLAIN, S.EPI_PARTS), "gate_up": (1, ks_gu, S.ROWS_GATE_UP, S.EPI_SILU_MUL),
            "down": (kp_down, ks_down, S.ROWS_PLAIN, S.EPI_PARTS), "head": (1, ks_head, S.ROWS_PLAIN, S.EPI_ARGMAX)}
    kp, ks, rowmap, epi = spec[name]
    wb = n * k // 32 * 18
    copies = max(1, min(copies, math.ceil(400e6 / wb)))
    x = torch.randn(k, device=device).to(BF16)
    key = torch.zeros(1, device=device, dtype=torch.int64)
    out = (torch.empty((kp, n), device=device, dtype=torch.float32) if epi == S.EPI_PARTS else
           torch.empty(n, device=device, dtype=BF16))
    progs = []
    for _ in range(copies):
        qs, d = _q4(n, k, device, gen)
        w = S.q4_pack_t16(qs, d, kp, rowmap, cfg.head_dim)
        del qs, d
        p = S.StepProgram(device)
        p.gemv(w, n, k, kp=kp, ks=ks, a=x, epi=epi, rowmap=rowmap, out=out, head_dim=cfg.head_dim,
               key=key if epi == S.EPI_ARGMAX else None)
        p.finalize()
        progs.append((p, p.io(key=key if epi == S.EPI_ARGMAX else None)))
    us = _time(lambda t: progs[t % copies][0].launch(progs[t % copies][1]), reps)
    byts = wb + 2 * k + (4 * kp if epi == S.EPI_PARTS else 2) * n
    return {"us": round(us, 3), "bytes": byts, "gbs": round(byts / us / 1e3, 1), "copies": copies, "kp": kp, "ks": ks}


def bench_step_q6_head(reps, copies, device, gen, n=131072, k=2560, ks=2):
    """The Q6_K LM head of the Spark checkpoint (tied embedding, 131072 x 2560) as a
    persistent-step GEMV stage with the argmax epilogue (T6 units)."""
    from . import step as S
    wb = S.t6_bytes(n, k)
    copies = max(1, min(copies, math.ceil(400e6 / wb)))
    x = torch.randn(k, device=device).to(BF16)
    key = torch.zeros(1, device=device, dtype=torch.int64)
    out = torch.empty(n, device=device, dtype=BF16)
    progs = []
    for _ in range(copies):
        blk = torch.randint(0, 256, (n * (k // 256), 210), device=device, dtype=torch.uint8, generator=gen)
        d = (torch.randn(n * (k // 256), device=device, generator=gen) * 2e-5).to(torch.float16)
        blk[:, 208:210] = d.view(torch.uint8).view(-1, 2)
        w = S.q6k_pack_t6(blk, n, k)
        del blk
        p = S.StepProgram(device)
        p.gemv(w, n, k, ks=ks, a=x, epi=S.EPI_ARGMAX, out=out, key=key, q6=True)
        p.finalize()
        progs.append((p, p.io(key=key)))
    us = _time(lambda t: progs[t % copies][0].launch(progs[t % copies][1]), reps)
    byts = wb + 2 * k + 2 * n
    return {"us": round(us, 3), "bytes": byts, "gbs": round(byts / us / 1e3, 1), "copies": copies, "ks": ks}


def bench_step_attn(ctx, reps, copies, device, gen, cfg):
    """The attention stage of the persistent decode-step kernel as its own launch
    (splits = CTAs / kv heads, distributed combine)."""
    from . import step as S
    nq, nkv, D, bs = cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim, cfg.block_size
    splits = S.attn_splits(cfg, S.num_ctas(), ctx)
    nblk = (ctx + bs - 1) // bs
    per = 2 * nblk * nkv * bs * D * 2
    copies = max(1, min(copies, math.ceil(400e6 / per)))
    q = torch.randn((nq, D), device=device).to(BF16)
    pos = torch.tensor([ctx - 1], device=device, dtype=torch.int64)
    progs = []
    for _ in range(copies):
        kc = torch.randn((nblk, nkv, bs, D), generator=gen, device=device).to(BF16)
        vc = torch.randn((nblk, nkv, bs, D), generator=gen, device=device).to(BF16)
        table = torch.randperm(nblk, device=device, generator=gen).to(torch.int32)
        kv_new = torch.zeros((2, nkv, D), device=device, dtype=BF16)
        po = torch.empty((splits, nq, D), device=device, dtype=torch.float32)
        pl = torch.empty((splits, nq), device=device, dtype=torch.float32)
        out = torch.empty((nq, D), device=device, dtype=BF16)
        hc = torch.zeros(nkv, device=device, dtype=torch.int32)
        p = S.StepProgram(device)
        p.attention(q=q, k_cache=kc, v_cache=vc, kv_new=kv_new, block_table=table, pos=pos, splits=splits,
                    max_split_tokens=S.max_split_tokens(ctx, splits), scale=cfg.attn_scale, part_o=po,
                    part_lse=pl, head_counters=hc, attn_out=out, nq=nq, nkv=nkv, head_dim=D, block_size=bs)
        p.finalize()
        progs.append((p, p.io()))
    us = _time(lambda t: progs[t % copies][0].launch(progs[t % copies][1]), reps)
    byts = 2 * ctx * nkv * D * 2 + 2 * nq * D * 2
    return {"us": round(us, 3), "bytes": byts, "gbs": round(byts / us / 1e3, 1), "splits": splits}


def bench_prefill_gemm(tokens, reps, device, gen, cfg, only=None):
    """The prefill GEMMs of one layer (qkv, o, gate_up, down) at ``tokens`` prompt tokens:
    the tcgen05 Q4_0 GEMM (``spark_q4_gemm_tc``) against cuBLAS over a cached bf16
    dequantization and against dequantize + cuBLAS.  µs per launch and TFLOP/s."""
    h, i = cfg.hidden_size, cfg.intermediate_size
    nh = cfg.num_q_heads + 2 * cfg.num_kv_heads
    shapes = {"qkv": (nh * cfg.head_dim, h), "o": (h, cfg.num_q_heads * cfg.head_dim), "gate_up": (2 * i, h),
              "down": (h, i)}
    res = {}
    for name, (n, k) in shapes.items():
        if only and name not in only:
            continue
        qs, d = _q4(n, k, device, gen)
        x = torch.randn((tokens, k), generator=gen, device=device).to(BF16)
        err = torch.zeros(1, dtype=torch.int32, device=device)
        wb = ops.q4_dequantize(qs, d)
        flop = 2.0 * tokens * n * k
        t_tc = _time(lambda _: ops.q4_gemm(x, qs, d, err), reps)
        t_blas = _time(lambda _: x @ wb.t(), reps)
        t_deq = _time(lambda _: x @ ops.q4_dequantize(qs, d).t(), reps)
        torch.cuda.synchronize()
        res[name] = {"shape": [tokens, n, k], "tc_us": round(t_tc, 1), "tc_tflops": round(flop / t_tc / 1e6, 1),
                     "cublas_cached_bf16_us": round(t_blas, 1), "dequant_cublas_us": round(t_deq, 1),
                     "error": int(err.item())}
        del qs, d, x, wb
    return res


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernels", default="gemv,qkv,o_proj,gate_up,down,head,attn")
    ap.add_argument("--reps", type=int, default=50)
    ap.add_argument("--copies", type=int, default=16)
    ap.add_argument("--ctx", default="2048,4096,6144")
    ap.add_argument("--splits", type=int, default=16)
    ap.add_argument("--tokens", type=int, default=2048, help="prompt tokens of --kernels prefill_gemm")
    ap.add_argument("--gemm-shapes", default="", help="prefill_gemm: a subset of qkv,o,gate_up,down")
    ap.add_argument("--direct", action="store_true", help="register-direct GEMV instead of the weight ring")
    ap.add_argument("--step", action="store_true",
                    help="stages of the persistent decode-step kernel (one cooperative launch each)")
    args = ap.parse_args(argv)
    device = torch.device("cuda")
    gen = torch.Generator(device=device).manual_seed(0)
    cfg = SparkConfig()
    ops.set_gemv_ring(not args.direct)
    out = {"path": "step" if args.step else ("direct" if args.direct else "ring")}
    cases = gemv_cases(cfg)
    for name in args.kernels.split(","):
        if name in cases:
            n, k, kind = cases[name]
            fn = bench_step_gemv if args.step else bench_gemv
            out[name] = fn(name, n, k, kind, args.reps, args.copies, device, gen, cfg)
        elif name == "prefill_gemm":
            out[name] = bench_prefill_gemm(args.tokens, args.reps, device, gen, cfg,
                                           args.gemm_shapes.split(",") if args.gemm_shapes else None)
        elif name == "head_q6" and args.step:
            out[name] = bench_step_q6_head(args.reps, args.copies, device, gen)
        elif name == "attn":
            for ctx in map(int, args.ctx.split(",")):
                out[f"attn_{ctx}"] = (bench_step_attn(ctx, args.reps, args.copies, device, gen, cfg) if args.step else
                                      bench_attn(ctx, args.splits, args.reps, args.copies, device, gen, cfg))
    out["device_error"] = ops.read_device_error()
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
