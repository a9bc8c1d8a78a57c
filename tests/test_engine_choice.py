"""Host-side choices that set what the benchmark runs: ``bench.resolve_mode`` (the decode
engine of ``--mode auto``) and ``spark_b200.model.chain_splits`` (the kernel chain's
attention split count).  Both are plain functions of the command line / context length,
checked here without a GPU."""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _args(**kw):
    base = dict(mode="auto", prompt=2048, steps=4096, warmup=16, tp=1, batch=1, model="synthetic-4b", splits=0)
    base.update(kw)
    return argparse.Namespace(**base)


@pytest.mark.parametrize("kw,world,want", [
    ({}, 1, "kernels"),                       # configs[2]: one batch-1 sequence, ctx 2048 -> 6143
    ({"steps": 20, "warmup": 5}, 1, "kernels"),
    ({"splits": 16}, 1, "kernels"),
    ({}, 2, "step"),                          # under torchrun: tensor parallelism
    ({"tp": 2}, 1, "step"),
    ({"batch": 4}, 1, "step"),                # configs[4] small batches
    ({"model": "spark-x26"}, 1, "step"),      # Spark layer features
    ({"prompt": 32768}, 1, "step"),           # beyond 16 wide-kernel splits
    ({"splits": 24}, 1, "step"),
    ({"mode": "step"}, 1, "step"),
    ({"mode": "kernels", "batch": 1}, 1, "kernels"),
])
def test_resolve_mode(kw, world, want):
    sys.path.insert(0, str(ROOT))
    import bench
    assert bench.resolve_mode(_args(**kw), world) == want


@pytest.mark.parametrize("max_seq,want", [(64, 16), (2069, 16), (6145, 16), (6400, 16), (6401, 51), (36865, 256)])
def test_chain_splits(max_seq, want):
    from spark_b200.model import chain_splits
    s = chain_splits(max_seq)
    assert s == want
    if s == 16:  # a split of the auto rule fits the wide attention kernel
        assert -(-max_seq // 16) <= 400
