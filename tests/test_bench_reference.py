"""The bench's reference arm (``bench.py --impl reference``: the C restatement of the
reference's CPU path, timed on the host cores) runs without a GPU and prints the
contract's JSON line: with the default ``--splits 0`` it takes the split count of the
engine the repo arm runs for the same command line (the kernel chain's 16 for one GPU,
``--mode step``: the persistent step's 18), and its ``e2e`` / ``cpu_baseline`` keys
describe the same run."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("mode,splits", [("auto", 16), ("step", 18)])  # step: 8 kv heads of 128 on 148 CTAs
def test_reference_arm_json_line(mode, splits):
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--layers", "1",
                          "--steps", "4", "--warmup", "3", "--mode", mode], cwd=ROOT, capture_output=True, text=True,
                         timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    d = json.loads(out.stdout.strip().splitlines()[-1])
    assert d["impl"] == "reference" and d["unit"] == "tokens/s" and d["value"] > 0
    assert d["config"]["splits"] == splits
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["h2d_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
