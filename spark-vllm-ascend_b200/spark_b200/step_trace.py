"""Per-stage timeline of one persistent decode step (the kernel's optional trace).

    python -m spark_b200.step_trace [--layers N] [--ctx C] [--model synthetic-4b|spark-x26]

Runs a synthetic model in persistent-step mode at context C, launches one traced step
(``SparkStepIO.trace``: globaltimer stamps per CTA and stage) and prints, per stage
kind, the median / max over CTAs of each phase averaged over layers, the barrier gap
(last CTA done -> first CTA starting the next stage) and how far ahead of the
consumers the producer started copying the stage's bytes.  GEMV phases: prologue
(loads, RMSNorm, staging), tasks, tail.  The prologue is further split into
loads (input vectors from L2), norm (sum of squares and 1/rms) and digits (fixed-point
staging of the input plus the CTA barrier).  Attention phases: ranges (each warp's
scores, softmax and P V over its token range), merge (the CTA's merge of the ranges),
publish (fused with o_proj: + waiting for the head's other splits), combine.
"""
from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from .config import SparkConfig
from .model import DecodeEngine, SyntheticWeights


def stage_kinds(num_layers: int) -> list[str]:
    return ["qkv", "attn", "o_proj", "gate_up", "down"] * num_layers + ["head"]


def summarize(t: np.ndarray, kinds: list[str]) -> dict:
    """t: int64 [ctas, stages, 8] trace stamps (ns)."""
    out: dict = {}
    prev_end = None
    for i, k in enumerate(kinds):
        c = t[:, i, :]
        act = c[:, 1] > 0
        c = c[act]
        d = out.setdefault(k, {"stages": 0})
        d["stages"] += 1
        ph = {"work": c[:, 2] - c[:, 1], "producer_lead": c[:, 1] - c[:, 3],
              # the producer's last copy of the stage issued this long before the stage began
              # (negative: issued after it began -- the stage waited for HBM / ring space)
              "producer_last_lead": c[:, 1] - c[:, 10]}
        if k == "attn":
            has = (c[:, 5] > 0) & (c[:, 7] > 0)  # splits with tokens (empty splits skip the phases)
            # ranges: the warps' scores / softmax / P V; merge: the CTA's merge of its ranges and
            # the split's partials; publish: counting the split (fused: and waiting for the
            # head's other splits); combine: the head's combine (fused: every CTA; else the
            # split that completed the head)
            ph.update({"ranges": c[has, 4] - c[has, 1], "merge": c[has, 5] - c[has, 4],
                       "publish": c[has, 6] - c[has, 5], "combine": c[has, 7] - c[has, 6],
                       "tail": c[has, 2] - c[has, 7]})
            # SM-cycle checkpoints of thread 0 (clock64): q + scores (of which the q loads), exp, P V, CTA barrier,
            # merge factors, merge outputs; combine: loads, weights, accumulation, staging
            raw = d.setdefault("raw", {})
            names = ["cyc_q_scores", "cyc_exp", "cyc_pv", "cyc_bar", "cyc_fac", "cyc_merge_out"]
            for q, nm in enumerate(names):
                ok = has & (c[:, 13 + q] > 0) & (c[:, 12 + q] > 0)
                if ok.any():
                    raw.setdefault(nm, []).append(float(np.median(c[ok, 13 + q] - c[ok, 12 + q])))
            ok = has & (c[:, 23] > 0) & (c[:, 12] > 0)  # q loads returned
            if ok.any():
                raw.setdefault("cyc_q_load", []).append(float(np.median(c[ok, 23] - c[ok, 12])))
            for q, nm in enumerate(["cyc_c_loads", "cyc_c_weights", "cyc_c_acc", "cyc_c_stage"]):
                ok = has & (c[:, 19 + q] > 0) & (c[:, 18 + q] > 0) & (c[:, 19 + q] >= c[:, 18 + q])
                if ok.any():
                    raw.setdefault(nm, []).append(float(np.median(c[ok, 19 + q] - c[ok, 18 + q])))
        else:
            has = c[:, 4] > 0
            ph.update({"prologue": c[has, 4] - c[has, 1], "tasks": c[has, 5] - c[has, 4],
                       "tail": c[has, 2] - c[has, 5]})
            fd = has & (c[:, 11] > 0)  # warp 0: time waiting for ring data; SM cycles per tile in its tasks
            ph["data_wait"] = c[fd, 9]
            raw = d.setdefault("raw", {})
            v = c[fd, 8] / c[fd, 11]
            if v.size:
                raw.setdefault("cycles_per_tile_warp0", []).append(float(np.median(v)))
                raw.setdefault("tiles_warp0", []).append(float(np.median(c[fd, 11])))
                # warp 0's SM cycles: in its GEMV tasks, after them (slice sums, epilogue,
                # slot release), and the whole task loop
                raw.setdefault("cyc_tasks", []).append(float(np.median(c[fd, 8])))
                raw.setdefault("cyc_post", []).append(float(np.median(c[fd, 12])))
                raw.setdefault("cyc_loop", []).append(float(np.median(c[fd, 13])))
            ld = has & (c[:, 6] > 0)  # staging split: loads | RMSNorm | digits + barrier
            nm = ld & (c[:, 7] > 0)
            ph["loads"] = c[ld, 6] - c[ld, 1]
            if nm.any():
                ph["norm"] = c[nm, 7] - c[nm, 6]
                ph["digits"] = c[nm, 4] - c[nm, 7]
            else:
                ph["digits"] = c[ld, 4] - c[ld, 6]
        for nm, v in ph.items():
            if v.size:
                acc = d.setdefault(nm, [0.0, 0.0])
                acc[0] += float(np.median(v))
                acc[1] += float(v.max())
        start, end = int(c[:, 1].min()), int(c[:, 2].max())
        if prev_end is not None:
            g = d.setdefault("barrier_gap", [0.0, 0.0])
            g[0] += start - prev_end
            g[1] += start - prev_end
        prev_end = end
    res = {}
    for k, d in out.items():
        n = d.pop("stages")
        raw = d.pop("raw", {})
        res[k] = {nm: {"median_us": round(v[0] / n / 1e3, 2), "max_us": round(v[1] / n / 1e3, 2)}
                  for nm, v in d.items()}
        res[k].update({nm: round(float(np.mean(v)), 1) for nm, v in raw.items()})  # medians over CTAs, mean over layers
        res[k]["stages"] = n
    return res


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=36)
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--model", choices=["synthetic-4b", "spark-x26"], default="synthetic-4b")
    args = ap.parse_args(argv)
    if args.model == "spark-x26":
        from .config import spark_x26_config
        cfg = spark_x26_config(num_layers=args.layers)
    else:
        cfg = SparkConfig(num_layers=args.layers)
    w = SyntheticWeights(cfg, device="cuda", seed=0)
    eng = DecodeEngine(w, max_seq_len=args.ctx + 64, num_blocks=(args.ctx + 64) // 128 + 8, use_graph=False)
    prog = eng.program
    eng.reset(args.ctx)
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
    tr = prog.trace_buffer()
    prog.launch(prog.io(error=eng.error, key=eng.key, token_out=eng.token, token_log=eng.token_log,
                        step=eng.step_idx, pos=eng.pos, trace=tr))
    torch.cuda.synchronize()
    t = tr.cpu().numpy().astype(np.int64)
    print(json.dumps({"layers": args.layers, "ctx": args.ctx, "ms_per_step": round(e0.elapsed_time(e1) / 20, 4),
                      "traced_step_us": round((t[:, -1, 2].max() - t[:, 0, 0].min()) / 1e3, 2),
                      "stages": summarize(t, stage_kinds(args.layers))}))


if __name__ == "__main__":
    main()
