"""GPU parity of the Q6_K path (the reference's Q6_K LM head over the tied embedding):

* ``spark_q6k_dequantize`` decodes gguf Q6_K super-blocks bit for bit like gguf 0.19.0
  (the committed golden vectors);
* the persistent step's Q6_K GEMV stage (T6 units, ``spark_q6k_pack_t6``) is bit-exact
  against the oracle's order (``orc_q6k_gemv_parts``) -- fp32 parts, bf16 outputs and
  the greedy argmax (that order's distance to a float64 dequantize-then-matmul is
  pinned on the CPU, tests/test_oracle.py);
* host validation refuses shapes the T6 layout cannot hold.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def u16(t):
    import torch
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def q6_rows(n: int, k: int, seed: int, d_std: float = 2e-4) -> np.ndarray:
    """n rows of random gguf Q6_K super-blocks (uint8 [n, k / 256 * 210])."""
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, size=(n * (k // 256), 210), dtype=np.uint8)
    d = (rng.standard_normal(b.shape[0]) * d_std).astype(np.float16)
    b[:, 208:210] = d.view(np.uint8).reshape(-1, 2)
    return b.reshape(n, -1)


def test_q6k_dequantize_matches_gguf_golden(cuda):
    import torch
    from spark_b200 import ops
    z = np.load(GOLDEN / "q6_k_gguf.npz")
    for name in ("normal", "edges", "rows"):
        got = ops.q6k_dequantize(torch.from_numpy(z[name + ".blocks"]).cuda()).cpu().numpy()
        want = z[name + ".deq"].reshape(-1)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), name


@pytest.mark.parametrize("n,k,kp,ks", [(16, 256, 1, 1), (64, 2560, 1, 2), (256, 2560, 1, 4), (160, 1024, 2, 2),
                                       (2560, 2560, 1, 2), (48, 512, 2, 1)])
def test_q6k_gemv_bitexact(cuda, oracle, n, k, kp, ks):
    import torch
    from spark_b200 import step
    rows = q6_rows(n, k, seed=n + k)
    w = step.q6k_pack_t6(torch.from_numpy(rows).cuda(), n, k, kp)
    x = (torch.randn(k, device="cuda") * torch.exp2(torch.randint(-6, 3, (k,), device="cuda").float())).to(
        torch.bfloat16)
    parts = torch.empty((kp, n), device="cuda", dtype=torch.float32)
    prog = step.StepProgram("cuda")
    prog.gemv(w, n, k, kp=kp, ks=ks, a=x, epi=step.EPI_PARTS, out=parts, q6=True)
    prog.finalize().launch(prog.io())
    want = oracle.q6k_gemv_parts(u16(x), rows, n, k, kp, ks)
    assert np.array_equal(parts.cpu().numpy().view(np.uint32), want.view(np.uint32))
    # (the order's distance to a float64 dequantize-then-matmul is pinned on the CPU:
    # tests/test_oracle.py::test_q6k_gemv_order_within_tolerance)


def test_q6k_head_argmax(cuda, oracle):
    """The tied-embedding head shape of the Spark checkpoint: 131072 x 2560, bf16 logits
    and the greedy token (lowest index on ties)."""
    import torch
    from spark_b200 import step
    n, k = 131072, 2560
    rows = q6_rows(n, k, seed=7)
    w = step.q6k_pack_t6(torch.from_numpy(rows).cuda(), n, k)
    x = torch.randn(k, device="cuda").to(torch.bfloat16)
    logits = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    key = torch.zeros(1, device="cuda", dtype=torch.int64)
    tok = torch.full((1,), -1, device="cuda", dtype=torch.int32)
    prog = step.StepProgram("cuda")
    prog.gemv(w, n, k, ks=2, a=x, epi=step.EPI_ARGMAX, out=logits, key=key, q6=True)
    prog.finalize().launch(prog.io(key=key, token_out=tok))
    torch.cuda.synchronize()
    want = oracle.parts_to_bf16(oracle.q6k_gemv_parts(u16(x), rows, n, k, 1, 2))
    assert np.array_equal(u16(logits), want)
    assert int(tok.item()) == oracle.argmax_bf16(want)


def test_q6k_rejects_bad_shapes(cuda):
    import torch
    from spark_b200 import step
    from spark_b200._lib import SparkError
    rows = torch.from_numpy(q6_rows(16, 512, seed=1)).cuda()
    with pytest.raises(SparkError):
        step.q6k_pack_t6(rows, 16, 512, 4)  # 128 columns per part: not whole super-blocks
    w = step.q6k_pack_t6(rows, 16, 512, 1)
    x = torch.randn(512, device="cuda").to(torch.bfloat16)
    y = torch.empty(16, device="cuda", dtype=torch.bfloat16)
    for kw in ({"ks": 3}, {"rowmap": step.ROWS_GATE_UP, "epi": step.EPI_SILU_MUL}):
        prog = step.StepProgram("cuda")
        prog.gemv(w, 16, 512, a=x, out=y, q6=True, **kw)
        with pytest.raises(SparkError):
            prog.finalize().launch(prog.io())
