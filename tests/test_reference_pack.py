"""Q4_0 format parity pinned to the reference's own repack code.

``tests/golden/ref_pack_q4.npz`` holds outputs of the reference's host functions
``unpack_q4`` (integration/weights.py:34-40: signed codes q - 8 and fp16 scales of each
gguf Q4_0 block) and ``pack`` (weights.py:42-54: the megakernel layout, tiles of m rows x
64 columns, two rows' codes per byte, bf16 scales), produced by importing the reference
tree (tests/golden/make_golden.py, ``make_ref_pack``).  These tests check that the qs / d
planes this library splits gguf blocks into carry exactly the reference's codes and
scales: the CPU split of the oracle, and (GPU) ``spark_q4_split_gguf`` on the device; and
that re-laying the planes in the reference's tile order reproduces ``pack``'s bytes.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"


def _fixture():
    return np.load(GOLDEN / "ref_pack_q4.npz")


def codes_from_planes(qs: np.ndarray, n: int, k: int) -> np.ndarray:
    """Signed codes q - 8 [n, k] from the nibble plane (byte j of a block: element j in
    the low nibble, element j + 16 in the high one)."""
    b = qs.reshape(n, k // 32, 16)
    lo = (b & 15).astype(np.int16) - 8
    hi = (b >> 4).astype(np.int16) - 8
    return np.concatenate((lo, hi), axis=-1).reshape(n, k).astype(np.int8)


def relay_reference_pack(qs: np.ndarray, d: np.ndarray, n: int, k: int, m: int) -> np.ndarray:
    """The planes in the reference megakernel's byte layout (weights.py:42-54): per tile
    of m rows, [K/64][m/2 row pairs][64] code bytes (row 2i in the low nibble, as the
    4-bit two's complement of q - 8), then [K/64][m/2][2 blocks][2 rows] bf16 scales."""
    q = codes_from_planes(qs, n, k).astype(np.int16)
    u = (q & 15).astype(np.uint8).reshape(n // m, m // 2, 2, k // 64, 64)
    codes = (u[:, :, 0] | (u[:, :, 1] << 4)).transpose(0, 2, 1, 3).reshape(n // m, m * k // 2)
    sc = d.view(np.float16).astype(np.float32).reshape(n // m, m // 2, 2, k // 64, 2)
    sc = sc.transpose(0, 3, 1, 4, 2)  # [tile][k64][row pair][block][row]
    bf = (sc.view(np.uint32) >> 16).astype(np.uint16).reshape(n // m, m * k // 32)
    assert np.array_equal((bf.astype(np.uint32) << 16).view(np.float32), sc.reshape(n // m, -1))
    return np.concatenate((codes, bf.view(np.uint8)), axis=1)


@pytest.mark.parametrize("case", ["gguf", "bf16"])
def test_oracle_split_matches_reference_unpack_q4(case):
    import oracle
    z = _fixture()
    blocks, q, s = z[f"{case}.blocks"], z[f"{case}.q"], z[f"{case}.s"]
    n, k = q.shape
    qs, d = oracle.q4_split(blocks.reshape(-1), n, k)
    assert np.array_equal(codes_from_planes(qs, n, k), q)
    assert np.array_equal(d.view(np.uint16), s.view(np.uint16))


@pytest.mark.parametrize("m", [8, 4])
def test_planes_relaid_equal_reference_pack(m):
    import oracle
    z = _fixture()
    blocks, q = z["bf16.blocks"], z["bf16.q"]
    n, k = q.shape
    qs, d = oracle.q4_split(blocks.reshape(-1), n, k)
    assert np.array_equal(relay_reference_pack(qs, d, n, k, m), z[f"bf16.pack{m}"])


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["gguf", "bf16"])
def test_device_split_matches_reference_unpack_q4(cuda, case):
    import torch
    from spark_b200 import ops
    z = _fixture()
    blocks, q, s = z[f"{case}.blocks"], z[f"{case}.q"], z[f"{case}.s"]
    n, k = q.shape
    qs, d = ops.q4_split_gguf(torch.from_numpy(blocks.reshape(-1).copy()).to(cuda), n, k)
    torch.cuda.synchronize()
    qs_h = qs.cpu().numpy()
    d_h = d.view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(codes_from_planes(qs_h, n, k), q)
    assert np.array_equal(d_h, s.view(np.uint16))
    if case == "bf16":
        for m in (8, 4):
            assert np.array_equal(relay_reference_pack(qs_h, d_h, n, k, m), z[f"bf16.pack{m}"])
