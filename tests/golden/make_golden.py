"""Generate the committed golden fixtures that pin the CPU oracle.

Run from the repository root in a container that has the third-party ``gguf``
package (version 0.19.0, the reference's pin in deployment/requirements.txt:5):

    python tests/golden/make_golden.py

Fixtures written next to this script:

* ``q4_0_gguf.npz`` -- seeded fp32 blocks and the bytes ``gguf.quants.quantize(...,
  Q4_0)`` produces for them, plus ``gguf.quants.dequantize`` of those bytes.  The
  reference calls the same functions at integration/weights.py:30 (dequantize)
  and tools/deployment/prepare_model.py:63; ``unpack_q4`` (weights.py:34-40)
  reads the same byte layout.  Cases cover N(0, 0.02) weights, wide dynamic
  range, all-zero blocks, ties between +max and -max, and a negative absmax.
* ``q6_k_gguf.npz`` -- seeded Q6_K super-blocks (256 weights, 210 bytes: 128 bytes of
  low nibbles, 64 of 2-bit high parts, 16 int8 sub-block scales, an fp16 scale) and
  ``gguf.quants.dequantize`` of them, the decode the reference's Q6_K head repack checks
  itself against (tools/deployment/prepare_head.py:23-26).  gguf 0.19.0 has no Q6_K
  quantizer, so the blocks are random bytes with chosen scales: N(0, 1e-3) fp16 scales,
  zero, negative and extreme (+-65504, subnormal) scales, sub-block scales -128 / 127,
  and a 131072 x 2560 row layout sample (10 blocks per row).
* ``slot_mapping_kat.npz`` -- the known-answer cases of
  tools/validation/test_slot_mapping.py:13-53 (block sizes {128, 256, 512, 1024},
  reversed tables ``arange(320).flip(0) + 400 i``, token counts {0, 1, 1025,
  2048, 4096} with offsets, and the graph-replay positions 4096/127/8192), with
  the expected slots computed by that test's own CPU formula (:26-28):
  ``table[pos // size] * size + pos % size``, -1 padding up to ``maximum``.
  Stored sparsely: only the first ``count`` entries (the rest are -1).
* ``ref_pack_q4.npz`` -- outputs of the reference's own host repack functions, imported
  from its source tree (``spark_vllm_ascend.integration.weights``: ``unpack_q4``,
  weights.py:34-40, and ``pack``, weights.py:42-54; pure numpy / torch): gguf Q4_0 block
  bytes, ``unpack_q4``'s signed codes and fp16 scales, and ``pack(q, s, m)`` for m = 8 and
  m = 4 (the tile heights the reference uses for qkv / o / gate_up and down,
  weights.py:62, 77).  ``pack`` asserts BF16-exact scales (weights.py:52), so the packed
  case uses blocks whose fp16 scales are bf16 values; the unpack case also covers the
  seeded N(0, 0.02) weights quantized by gguf.  Needs the reference tree: the ``src``
  directory of its checkout in ``SPARK_REFERENCE_SRC``; skipped when that is unset.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def q4_cases() -> dict[str, np.ndarray]:
    rng = np.random.default_rng(1234)
    cases = {}
    cases["normal"] = (rng.standard_normal((64, 512)) * 0.02).astype(np.float32)
    wide = rng.standard_normal((16, 256)).astype(np.float32)
    wide *= np.exp2(rng.integers(-20, 12, size=(16, 256))).astype(np.float32)
    cases["wide"] = wide
    z = (rng.standard_normal((4, 128)) * 0.5).astype(np.float32)
    z[0, :32] = 0.0
    z[1, 32:64] = 0.0
    z[2, 64:96] = -0.0
    cases["zeros"] = z
    t = (rng.standard_normal((4, 128)) * 0.1).astype(np.float32)
    t[0, 3], t[0, 17] = 0.5, -0.5     # tie: +max first
    t[1, 5], t[1, 9] = -0.75, 0.75    # tie: -max first
    t[2, 40], t[2, 41] = -2.0, 1.0    # negative absmax
    t[3, :32] = np.linspace(-1, 1, 32, dtype=np.float32)
    cases["ties"] = t
    big = (rng.standard_normal((2, 64)) * 3000.0).astype(np.float32)
    cases["large"] = big
    return cases


def make_q4() -> None:
    from gguf import GGMLQuantizationType as T
    from gguf import quants

    out = {}
    for name, w in q4_cases().items():
        blocks = quants.quantize(w, T.Q4_0)
        deq = quants.dequantize(blocks, T.Q4_0)
        out[f"{name}.w"] = w
        out[f"{name}.blocks"] = np.ascontiguousarray(blocks, dtype=np.uint8)
        out[f"{name}.deq"] = np.ascontiguousarray(deq, dtype=np.float32)
    np.savez_compressed(HERE / "q4_0_gguf.npz", **out)


def q6k_blocks(rng, n: int) -> np.ndarray:
    """n random Q6_K blocks (uint8 [n, 210]) with fp16 scales ~ N(0, 1e-3)."""
    b = rng.integers(0, 256, size=(n, 210), dtype=np.uint8)
    d = (rng.standard_normal(n) * 1e-3).astype(np.float16)
    b[:, 208:210] = d.view(np.uint8).reshape(n, 2)
    return b


def make_q6k() -> None:
    from gguf import GGMLQuantizationType as T
    from gguf import quants

    rng = np.random.default_rng(4321)
    cases = {"normal": q6k_blocks(rng, 64)}
    e = q6k_blocks(rng, 8)
    d = np.array([0.0, -0.0, 65504.0, -65504.0, 6e-8, -3e-5, 1.0, -0.5], np.float16)
    e[:, 208:210] = d.view(np.uint8).reshape(8, 2)
    e[0:4, 192:208] = np.array([-128, 127] * 8, np.int8).view(np.uint8)
    cases["edges"] = e
    cases["rows"] = q6k_blocks(rng, 40)  # 4 rows of K = 2560 (10 blocks per row)
    out = {}
    for name, blocks in cases.items():
        out[f"{name}.blocks"] = np.ascontiguousarray(blocks)
        out[f"{name}.deq"] = np.ascontiguousarray(quants.dequantize(blocks, T.Q6_K), dtype=np.float32)
    np.savez_compressed(HERE / "q6_k_gguf.npz", **out)


def make_slots() -> None:
    maximum = 32768
    sizes = [128, 256, 512, 1024]
    tables = [np.arange(320, dtype=np.int32)[::-1] + i * 400 for i in range(4)]
    cases = [(c, o) for c, o in [(0, 0), (1, 127), (1025, 63), (2048, 3072), (4096, 0)]]
    cases += [(1, 4096), (1, 127), (1, 8192)]
    out = {"maximum": np.int64(maximum), "sizes": np.array(sizes, np.int64),
           "tables": np.stack(tables), "cases": np.array(cases, np.int64)}
    for ci, (count, offset) in enumerate(cases):
        pos = np.arange(count, dtype=np.int64) + offset
        for gi, (table, size) in enumerate(zip(tables, sizes)):
            expected = table[pos // size].astype(np.int64) * size + pos % size
            out[f"case{ci}.group{gi}"] = expected
    np.savez_compressed(HERE / "slot_mapping_kat.npz", **out)


class _GgufTensor:
    """The attributes of a gguf ReaderTensor that ``unpack_q4`` reads."""

    def __init__(self, blocks: np.ndarray, n: int, k: int):
        self.name = "synthetic.weight"
        self.tensor_type = 2  # GGMLQuantizationType.Q4_0
        self.shape = np.array([k, n], dtype=np.uint64)  # gguf order: innermost first
        self.data = blocks.reshape(n, k // 32 * 18)


def ref_pack_blocks(rng, n: int, k: int) -> np.ndarray:
    """Q4_0 blocks [n, k/32, 18] with random nibbles and fp16 scales that are bf16 values
    (the reference's pack requires BF16-exact scales)."""
    d32 = (rng.standard_normal((n, k // 32)) * 2e-3).astype(np.float32)
    d_bf = (d32.view(np.uint32) & 0xFFFF0000).view(np.float32)  # truncate to bf16
    d16 = d_bf.astype(np.float16)
    assert np.array_equal(d16.astype(np.float32), d_bf)
    b = np.empty((n, k // 32, 18), np.uint8)
    b[:, :, :2] = d16.view(np.uint8).reshape(n, k // 32, 2)
    b[:, :, 2:] = rng.integers(0, 256, size=(n, k // 32, 16), dtype=np.uint8)
    return b


def make_ref_pack() -> bool:
    import os
    import sys
    src = os.environ.get("SPARK_REFERENCE_SRC", "")
    if not src or not Path(src, "spark_vllm_ascend", "integration", "weights.py").exists():
        print("reference tree not found: ref_pack_q4.npz not regenerated")
        return False
    sys.path.insert(0, src)
    from gguf import GGMLQuantizationType as T
    from gguf import quants
    from spark_vllm_ascend.integration.weights import pack, unpack_q4

    rng = np.random.default_rng(2468)
    out = {}
    n, k = 64, 512
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    blocks = np.ascontiguousarray(quants.quantize(w, T.Q4_0), dtype=np.uint8).reshape(n, k // 32, 18)
    q, s = unpack_q4(_GgufTensor(blocks, n, k))
    out.update({"gguf.blocks": blocks, "gguf.q": q, "gguf.s": s})
    n, k = 32, 256
    blocks = ref_pack_blocks(rng, n, k)
    q, s = unpack_q4(_GgufTensor(blocks, n, k))
    out.update({"bf16.blocks": blocks, "bf16.q": q, "bf16.s": s,
                "bf16.pack8": pack(q, s, 8), "bf16.pack4": pack(q, s, 4)})
    np.savez_compressed(HERE / "ref_pack_q4.npz", **out)
    return True


if __name__ == "__main__":
    make_q4()
    make_q6k()
    make_slots()
    make_ref_pack()
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)
