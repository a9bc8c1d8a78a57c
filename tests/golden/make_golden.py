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
* ``slot_mapping_kat.npz`` -- the known-answer cases of
  tools/validation/test_slot_mapping.py:13-53 (block sizes {128, 256, 512, 1024},
  reversed tables ``arange(320).flip(0) + 400 i``, token counts {0, 1, 1025,
  2048, 4096} with offsets, and the graph-replay positions 4096/127/8192), with
  the expected slots computed by that test's own CPU formula (:26-28):
  ``table[pos // size] * size + pos % size``, -1 padding up to ``maximum``.
  Stored sparsely: only the first ``count`` entries (the rest are -1).
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


if __name__ == "__main__":
    make_q4()
    make_slots()
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)
