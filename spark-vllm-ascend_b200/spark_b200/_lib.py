"""ctypes binding of ``libspark_b200.so`` (the C ABI in include/spark_b200.h).

There is no fallback: if the shared library is missing or cannot be loaded,
``lib()`` raises, so no caller can silently run something other than the sm_100a
kernels.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libspark_b200.so"
_lib = None

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F = ctypes.c_float

# name -> argument types (all return int status)
SIGNATURES: dict[str, list] = {
    "spark_q4_quantize": [_P, _I64, _I64, _P, _P, _P],
    "spark_q4_split_gguf": [_P, _I64, _I64, _P, _P, _P],
    "spark_q4_dequantize_bf16": [_P, _P, _I64, _I64, _P, _P],
    "spark_q4_gemm_tc": [_P, _P, _P, _P, _I, _I, _I, _P, _I64, _P],
    "spark_q4_gemv": [_P, _P, _P, _P, _I, _I, _I, _P],
    "spark_rmsnorm_q4_gemv": [_P, _P, _P, _F, _P, _P, _P, _P, _I, _I, _P],
    "spark_rmsnorm_gate_up_silu": [_P, _P, _P, _F, _P, _P, _P, _P, _I, _I, _P],
    "spark_qkv_rope_kvstore": [_P, _P, _P, _P, _P, _F, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _I, _P, _P, _P,
                               _P],
    "spark_attn_splitkv": [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _F, _P, _P, _P, _P],
    "spark_attn_combine": [_P, _P, _I, _I, _I, _P, _P],
    "spark_attn_decode_noalloc": [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _F, _P, _P, _P],
    "spark_attn_decode": [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _F, _P, _P, _P, _P, _P, _P],
    "spark_rmsnorm_q4_head_argmax": [_P, _P, _P, _F, _P, _P, _P, _I, _I, _P, _P],
    "spark_decode_finalize": [_P, _P, _P, _P, _P, _P],
    "spark_add_rmsnorm": [_P, _P, _P, _F, _I, _P, _P, _P],
    "spark_silu_mul": [_P, _P, _I64, _P, _P],
    "spark_rope_neox": [_P, _I, _I, _P, _P, _P],
    "spark_add_rmsnorm_rows": [_P, _P, _P, _F, _I, _I, _P, _P, _P],
    "spark_rope_neox_rows": [_P, _I64, _I, _I, _I, _I, _P, _I64, _P],
    "spark_act_mul_rows": [_P, _I, _I, _P, _P, _P],
    "spark_slot_mapping": [_I64, _I64, _P, _P, _P, _I64, _P, _P],
    "spark_set_pdl": [_I],
    "spark_set_gemv_ring": [_I],
    "spark_read_device_error": [_P, _I],
    "spark_kv_store": [_P, _P, _P, _I64, _I, _I, _I, _P, _P, _P],
    "spark_t16_bytes": [_I, _I, _I],
    "spark_q4_pack_t16": [_P, _P, _I, _I, _I, _I, _I, _P, _P],
    "spark_step_ring_bytes": [],
    "spark_step_ring_bytes_batch": [_I],
    "spark_step_num_ctas": [],
    "spark_step_run": [_P, _P, _I, _P, _P],
    "spark_t6_bytes": [_I, _I],
    "spark_q6k_pack_t6": [_P, _I, _I, _I, _P, _P],
    "spark_q6k_dequantize": [_P, _I64, _P, _P],
    "spark_window_alloc": [ctypes.c_uint64, ctypes.POINTER(_P)],
    "spark_window_free": [_P],
    "spark_ipc_handle": [_P, _P],
    "spark_ipc_open": [_P, ctypes.POINTER(_P)],
    "spark_ipc_close": [_P],
}
# entry points whose return value is a quantity, not a status
RESTYPES = {"spark_t16_bytes": _I64, "spark_t6_bytes": _I64}


class SparkStage(ctypes.Structure):
    """Mirror of ``SparkStage`` in include/spark_b200.h (288 bytes)."""

    _fields_ = [(n, ctypes.c_int32) for n in (
        "kind", "pro", "epi", "rowmap", "n", "k", "kp", "ks", "units", "rot", "wait", "norm", "a_parts",
        "block_size", "nq", "nkv", "head_dim", "splits", "max_split_tokens", "xchg")] + [
        (n, ctypes.c_float) for n in ("eps", "inv_k", "scale")] + [("row0", ctypes.c_int32)] + [
        (n, _P) for n in (
            "w", "a", "b", "embed", "token", "gamma", "res_out", "out", "cos_sin", "pos", "block_table", "k_cache",
            "v_cache", "q", "kv_new", "key", "part_o", "part_lse", "head_counters", "attn_out")] + [
        ("rotary_dim", ctypes.c_int32), ("window", ctypes.c_int32), ("table", _P), ("gate", _P),
        ("batch", ctypes.c_int32), ("bt_stride", ctypes.c_int32)]


class SparkStepIO(ctypes.Structure):
    """Mirror of ``SparkStepIO`` in include/spark_b200.h."""

    _fields_ = [(n, _P) for n in ("counters", "error", "key", "token_out", "token_log", "step", "pos", "trace",
                                  "peer_windows", "window")] + [
        ("window_bytes", ctypes.c_uint64), ("tp_size", ctypes.c_int32), ("tp_rank", ctypes.c_int32)]


assert ctypes.sizeof(SparkStage) == 288


class SparkError(RuntimeError):
    """A C-ABI entry point returned a non-zero status."""

    def __init__(self, fn: str, status: int, text: str):
        super().__init__(f"{fn} failed with status {status}: {text}")
        self.fn = fn
        self.status = status


def library_path() -> Path:
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            raise RuntimeError(
                f"spark_b200 CUDA library not found at {_LIB_PATH}; build it with "
                "`python spark-vllm-ascend_b200/build.py` (there is no CPU fallback)")
        L = ctypes.CDLL(str(_LIB_PATH))
        for name, args in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = RESTYPES.get(name, _I)
            fn.argtypes = args
        L.spark_status_string.restype = ctypes.c_char_p
        L.spark_status_string.argtypes = [_I]
        L.spark_version.restype = _I
        L.spark_version.argtypes = []
        _lib = L
    return _lib


def call(name: str, *args) -> None:
    """Call an entry point and raise SparkError on a non-zero status."""
    L = lib()
    status = getattr(L, name)(*args)
    if status != 0:
        raise SparkError(name, status, L.spark_status_string(status).decode())
