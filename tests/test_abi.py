"""CPU checks of the C ABI: the library builds, loads without a GPU and exports
every entry point that include/spark_b200.h declares; the ctypes table matches.
No compute call is made here."""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "spark_b200.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(spark_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def libpath():
    import spark_b200
    from spark_b200._lib import library_path

    spark_b200.ensure_built()
    return library_path()


def test_header_declares_entry_points():
    syms = declared_symbols()
    for must in ("spark_q4_gemv", "spark_attn_splitkv", "spark_attn_combine", "spark_qkv_rope_kvstore",
                 "spark_rmsnorm_gate_up_silu", "spark_rmsnorm_q4_head_argmax", "spark_slot_mapping"):
        assert must in syms


def test_library_exports_every_declared_symbol(libpath):
    out = subprocess.run(["nm", "-D", "--defined-only", str(libpath)], capture_output=True, text=True, check=True)
    exported = set(re.findall(r"\sT\s(spark_[a-z0-9_]+)$", out.stdout, flags=re.M))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, missing


def test_library_loads_and_reports_without_gpu(libpath):
    from spark_b200 import _lib

    L = _lib.lib()
    assert L.spark_version() >= 100
    assert L.spark_status_string(0) == b"ok"
    assert b"unsupported" in L.spark_status_string(2)


def test_ctypes_table_covers_header():
    from spark_b200._lib import SIGNATURES

    syms = set(declared_symbols()) - {"spark_version", "spark_status_string"}
    assert syms <= set(SIGNATURES), sorted(syms - set(SIGNATURES))


def test_host_validation_rejects_bad_shapes_before_launch(libpath):
    """Shape / pointer checks run on the host: no device work is issued."""
    from spark_b200 import _lib

    L = _lib.lib()
    fake = ctypes.c_void_p(0x1000)  # never dereferenced: validation fails first
    # n odd
    assert L.spark_q4_gemv(fake, fake, fake, fake, 3, 64, 1, None) == 2
    # k not a multiple of 32
    assert L.spark_q4_gemv(fake, fake, fake, fake, 4, 48, 1, None) == 2
    # batch out of range
    assert L.spark_q4_gemv(fake, fake, fake, fake, 4, 64, 9, None) == 2
    # null weights
    assert L.spark_q4_gemv(fake, None, fake, fake, 4, 64, 1, None) == 1
    # misaligned nibble plane
    assert L.spark_q4_gemv(fake, ctypes.c_void_p(0x1001), fake, fake, 4, 64, 1, None) == 3
    # attention: unsupported head_dim / group size, too-long splits
    args = [fake, fake, fake, fake, fake, None]
    assert L.spark_attn_splitkv(*args, 32, 8, 64, 128, 16, 256, ctypes.c_float(0.1), fake, fake, None, None) == 2
    assert L.spark_attn_splitkv(*args, 32, 4, 128, 128, 16, 256, ctypes.c_float(0.1), fake, fake, None, None) == 2
    assert L.spark_attn_splitkv(*args, 32, 8, 128, 128, 16, 4096, ctypes.c_float(0.1), fake, fake, None, None) == 5
    assert L.spark_slot_mapping(10, 5, fake, fake, fake, 128, fake, None) == 2
    # tensor-core prefill GEMM: K a multiple of 256, 16-byte aligned x / qs / d, a status word
    err = ctypes.c_void_p(0x2000)
    assert L.spark_q4_gemm_tc(fake, fake, fake, fake, 4, 128, 320, err, -1, None) == 2
    assert L.spark_q4_gemm_tc(fake, fake, fake, fake, 0, 128, 256, err, -1, None) == 2
    assert L.spark_q4_gemm_tc(fake, fake, fake, fake, 4, 128, 256, None, -1, None) == 1
    assert L.spark_q4_gemm_tc(fake, fake, ctypes.c_void_p(0x1008), fake, 4, 128, 256, err, -1, None) == 3
    # prefill row kernels: shapes
    assert L.spark_add_rmsnorm_rows(fake, None, fake, ctypes.c_float(1e-6), 4, 16384, None, fake, None) == 2
    assert L.spark_act_mul_rows(fake, 0, 64, None, fake, None) == 2
