"""Per-stage timeline of one persistent decode step (the kernel's optional trace).

    python -m spark_b200.step_trace [--layers N] [--ctx C] [--model synthetic-4b|spark-x26]

Runs a synthetic model in persistent-step mode at context C, launches one traced step
(``SparkStepIO.trace``: globaltimer stamps per CTA and stage) and prints, per stage
kind, the median / max over CTAs of each phase averaged over layers, the barrier gap
(last CTA done -> first CTA starting the next stage) and how far ahead of the
consumers the producer started copying the stage's bytes.  GEMV phases: prologue
(loads, RMSNorm, staging), tasks, tail.  The prologue is further split into
loads (input vectors from L2), norm (sum of squares and 1/rms) and digits (fixed-point
staging of the input plus the CTA barrier).  Attention phases: scores, softmax, PV,
publish (+ waiting for the head's other splits), combine.
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
        ph = {"work": c[:, 2] - c[:, 1], "producer_lead": c[:, 1] - c[:, 3]}
        if k == "attn":
            has = (c[:, 7] > 0) & (c[:, 6] > 0)  # splits with tokens (empty splits skip the phases)
            ph.update({"scores": c[has, 4] - c[has, 1], "softmax": c[has, 5] - c[has, 4], "pv": c[has, 6] - c[has, 5],
                       "publish_wait": c[has, 7] - c[has, 6], "combine": c[has, 2] - c[has, 7]})
        else:
            has = c[:, 4] > 0
            ph.update({"prologue": c[has, 4] - c[has, 1], "tasks": c[has, 5] - c[has, 4],
                       "tail": c[has, 2] - c[has, 5]})
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
        res[k] = {nm: {"median_us": round(v[0] / n / 1e3, 2), "max_us": round(v[1] / n / 1e3, 2)}
                  for nm, v in d.items()}
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
