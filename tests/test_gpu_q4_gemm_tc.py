"""GPU parity of the tensor-core Q4_0 prefill GEMM (``spark_q4_gemm_tc``, tcgen05.mma with
the weight tile dequantized in shared memory) against the same product in fp32 over the
bf16 dequantization (``spark_q4_dequantize_bf16``, the reference's
``dequantize(...).bfloat16()`` weights, integration/weights.py:28-31) and against the
cuBLAS bf16 matmul the prefill used before.  Both accumulate in fp32 over identical bf16
operands, so they differ only by summation order: tolerance rel 1e-2 + abs 1e-3 of the
row scale, and at least 99 % of outputs bit-identical to cuBLAS's.
"""
from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu

SHAPES = [  # (tokens, rows, K)
    (1, 128, 256),
    (77, 200, 2560),
    (128, 256, 4096),
    (300, 6144, 2560),
    (129, 2560, 9728),
]


def _planes(n, k, seed):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    qs = torch.randint(0, 256, (n, k // 2), generator=g, device="cuda", dtype=torch.int32).to(torch.uint8)
    d = (torch.rand((n, k // 32), generator=g, device="cuda") * 0.01 + 1e-4).to(torch.float16)
    return qs, d


@pytest.mark.parametrize("t,n,k", SHAPES)
def test_q4_gemm_tc_matches_fp32_and_cublas(cuda, t, n, k):
    import torch
    from spark_b200 import ops
    qs, d = _planes(n, k, seed=t * 7 + n)
    g = torch.Generator(device="cuda").manual_seed(n + k)
    x = torch.randn((t, k), generator=g, device="cuda").to(torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    y = ops.q4_gemm(x, qs, d, err)
    w = ops.q4_dequantize(qs, d)
    ref = x.float() @ w.float().t()
    blas = x @ w.t()
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert y.shape == (t, n) and y.dtype == torch.bfloat16
    scale = ref.abs().amax(dim=1, keepdim=True).clamp_min(1e-6)
    diff = (y.float() - ref).abs()
    assert bool((diff <= 1e-2 * ref.abs() + 1e-3 * scale).all()), float((diff / scale).max())
    same = (y.view(torch.int16) == blas.view(torch.int16)).float().mean().item()
    assert same >= 0.99, same


@pytest.mark.parametrize("n,k", [(200, 256), (384, 2560)])
def test_q4_gemm_tc_identity_is_bit_exact_dequant(cuda, n, k):
    """x = the identity: every output is one product W[n][t] * 1, so y must equal the
    transposed bf16 dequantization exactly (scales of either sign, q = 0..15).  Compared
    as values: a -0.0 weight (negative scale, q = 8) sums with the +0.0 products of the
    other columns to +0.0, so only the sign of zero may differ."""
    import torch
    from spark_b200 import ops
    qs, d = _planes(n, k, seed=n)
    d = torch.where(torch.arange(d.numel(), device="cuda").reshape(d.shape) % 3 == 0, -d, d)
    x = torch.eye(k, dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    y = ops.q4_gemm(x, qs, d, err)
    w = ops.q4_dequantize(qs, d)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(y.float(), w.t().float())
    nz = w.t() != 0
    assert torch.equal(y.view(torch.int16)[nz], w.t().contiguous().view(torch.int16)[nz])


def test_q4_gemm_tc_rejects_bad_shapes(cuda):
    import torch
    from spark_b200 import ops
    qs, d = _planes(128, 320, seed=1)  # K = 320: not a multiple of 256
    x = torch.zeros((4, 320), dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(Exception):
        ops.q4_gemm(x, qs, d, err)


def test_q4_gemm_tc_wait_timeout_reports_and_recovers(cuda):
    """A wait limit of 0 ns makes the first unfinished wait give up: the kernel must
    return (no hang), report 1 in the caller's status word (not 2: the issued MMAs drained
    and the tensor memory was freed), and the next call with the default limit must
    match the dequantize + fp32 product again on the same context."""
    import torch
    from spark_b200 import ops
    t, n, k = 256, 512, 4096  # 64 K steps per CTA: waits on in-flight MMAs are certain
    qs, d = _planes(n, k, seed=5)
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn((t, k), generator=g, device="cuda").to(torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.q4_gemm(x, qs, d, err, wait_ns=0)
    torch.cuda.synchronize()
    assert int(err.item()) == 1
    err.zero_()
    y = ops.q4_gemm(x, qs, d, err)
    w = ops.q4_dequantize(qs, d)
    ref = x.float() @ w.float().t()
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    scale = ref.abs().amax(dim=1, keepdim=True).clamp_min(1e-6)
    diff = (y.float() - ref).abs()
    assert bool((diff <= 1e-2 * ref.abs() + 1e-3 * scale).all()), float((diff / scale).max())
