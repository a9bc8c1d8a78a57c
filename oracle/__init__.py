"""CPU oracle for the Spark decode hot path -- TEST INFRASTRUCTURE ONLY.

This package wraps ``spark_oracle.c`` (a plain-C restatement of the reference
algorithm, see that file's header for the reference anchors) with ctypes and
numpy.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline legs may import it; the product package ``spark_b200`` never does, and
it fails loudly when its CUDA library is missing instead of falling back here.

All bf16 arrays are numpy ``uint16`` bit patterns; fp16 scales are ``uint16``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "libspark_oracle.so"
_lib = None

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float


def build(force: bool = False) -> Path:
    """Compile the oracle with its Makefile (gcc, no GPU needed)."""
    if force or not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < (_HERE / "spark_oracle.c").stat().st_mtime:
        subprocess.run(["make", "-C", str(_HERE), "-s"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        flags = Path("/proc/cpuinfo").read_text() if Path("/proc/cpuinfo").exists() else ""
        if " fma " not in flags or " avx2 " not in flags:
            raise RuntimeError("the oracle is compiled for x86-64 with AVX2+FMA; this CPU lacks them")
        L = ctypes.CDLL(str(_LIB_PATH))
        sig = {
            "orc_exp": (_F, [_F]),
            "orc_log": (_F, [_F]),
            "orc_q4_quantize": (None, [_P, _I64, _I64, _P, _P]),
            "orc_q4_split": (None, [_P, _I64, _I64, _P, _P]),
            "orc_q4_join": (None, [_P, _P, _I64, _I64, _P]),
            "orc_q4_dequantize": (None, [_P, _P, _I64, _I64, _P]),
            "orc_q4_gemv_f32": (None, [_P, _P, _P, _I64, _I64, _I, _P]),
            "orc_q4_gemv": (None, [_P, _P, _P, _I64, _I64, _I, _P]),
            "orc_q4_stage_x": (None, [_P, _I64, _P, _P, _P]),
            "orc_add_rmsnorm": (None, [_P, _P, _P, _I, _F, _P, _P]),
            "orc_rope_neox": (None, [_P, _I, _I, _P]),
            "orc_silu_mul": (None, [_P, _P, _I64, _P]),
            "orc_slot_mapping": (None, [_I64, _I64, _I64, _I64, _P, _P, _I64, _P]),
            "orc_split_tokens": (_I64, [_I64, _I]),
            "orc_t16_gemv_parts": (None, [_P, _P, _P, _I64, _I64, _I, _I, _P]),
            "orc_q6k_dequantize": (None, [_P, _I64, _P]),
            "orc_q6k_gemv_parts": (None, [_P, _P, _I64, _I64, _I, _I, _P]),
            "orc_t16_gemv": (None, [_P, _P, _P, _I64, _I64, _I, _I, _P]),
            "orc_parts_to_bf16": (None, [_P, _I, _I64, _P]),
            "orc_attn_split_w": (None, [_P, _P, _P, _P, _I64, _I, _I, _I, _I, _I, _F, _I, _P, _P]),
            "orc_attn_split": (None, [_P, _P, _P, _P, _I64, _I, _I, _I, _I, _I, _F, _P, _P]),
            "orc_attn_combine": (None, [_P, _P, _I, _I, _I, _P]),
            "orc_attn_split_x": (None, [_P, _P, _P, _P, _I64, _I, _I, _I, _I, _I, _F, _I, _I, _P, _P]),
            "orc_attn_combine_g": (None, [_P, _P, _I, _I, _I, _P, _P]),
            "orc_rope_partial": (None, [_P, _I, _I, _I, _P]),
            "orc_gelu_mul": (None, [_P, _P, _I64, _P, _P]),
            "orc_sigmoid_bf16": (None, [_P, _I64, _P]),
            "orc_argmax_bf16": (_I64, [_P, _I64]),
            "orc_decode_step": (_I64, [_P, _P, _P, _P, _P, _I64, _P, _I64, _I64, _F, _F, _P]),
            "orc_decode_layer": (None, [_P, _P, _P, _P, _P, _P, _I64, _F, _F, _P, _P, _I]),
            "orc_decode_head": (_I64, [_P, _P, _P, _P, _F, _P]),
            "orc_set_threads": (None, [_I]),
            "orc_get_threads": (_I, []),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data


# ----------------------------------------------------------------- bf16 helpers
def f32_to_bf16(a) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bits (uint16)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FFF
    return r


def bf16_to_f32(b) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ----------------------------------------------------------------- Q4_0
def q4_quantize(w: np.ndarray):
    """fp32 [rows, k] -> (qs uint8 [rows, k/2], d uint16 [rows, k/32]) (gguf Q4_0)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, k = w.shape
    assert k % 32 == 0
    qs = np.empty((rows, k // 2), np.uint8)
    d = np.empty((rows, k // 32), np.uint16)
    lib().orc_q4_quantize(_p(w), rows, k, _p(qs), _p(d))
    return qs, d


def q4_split(blocks: np.ndarray, rows: int, k: int):
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    qs = np.empty((rows, k // 2), np.uint8)
    d = np.empty((rows, k // 32), np.uint16)
    lib().orc_q4_split(_p(blocks), rows, k, _p(qs), _p(d))
    return qs, d


def q4_join(qs: np.ndarray, d: np.ndarray) -> np.ndarray:
    rows, k = qs.shape[0], qs.shape[1] * 2
    out = np.empty((rows, k // 32 * 18), np.uint8)
    lib().orc_q4_join(_p(np.ascontiguousarray(qs)), _p(np.ascontiguousarray(d)), rows, k, _p(out))
    return out


def q4_dequantize(qs: np.ndarray, d: np.ndarray) -> np.ndarray:
    rows, k = qs.shape[0], qs.shape[1] * 2
    w = np.empty((rows, k), np.float32)
    lib().orc_q4_dequantize(_p(np.ascontiguousarray(qs)), _p(np.ascontiguousarray(d)), rows, k, _p(w))
    return w


def q4_gemv(x_bf16: np.ndarray, qs: np.ndarray, d: np.ndarray) -> np.ndarray:
    """x bf16 [batch, k] (uint16) -> y bf16 [batch, n] in the canonical order."""
    x = np.ascontiguousarray(np.atleast_2d(x_bf16), dtype=np.uint16)
    n, k = qs.shape[0], qs.shape[1] * 2
    batch = x.shape[0]
    assert x.shape[1] == k
    y = np.empty((batch, n), np.uint16)
    lib().orc_q4_gemv(_p(x), _p(np.ascontiguousarray(qs)), _p(np.ascontiguousarray(d)), n, k, batch, _p(y))
    return y


def q4_stage_x(x_f32: np.ndarray):
    """Per-block 16-bit fixed point of x: (X int16 [k], sx fp32 [k/32], C int32 [k/32])."""
    x = np.ascontiguousarray(x_f32, dtype=np.float32)
    k = x.size
    X = np.empty(k, np.int16)
    sx = np.empty(k // 32, np.float32)
    C = np.empty(k // 32, np.int32)
    lib().orc_q4_stage_x(_p(x), k, _p(X), _p(sx), _p(C))
    return X, sx, C


def q4_gemv_f32(x_f32: np.ndarray, qs: np.ndarray, d: np.ndarray) -> np.ndarray:
    """Unrounded fp32 sums (same order) -- used to study rounding boundaries."""
    x = np.ascontiguousarray(np.atleast_2d(x_f32), dtype=np.float32)
    n, k = qs.shape[0], qs.shape[1] * 2
    y = np.empty((x.shape[0], n), np.float32)
    lib().orc_q4_gemv_f32(_p(x), _p(np.ascontiguousarray(qs)), _p(np.ascontiguousarray(d)), n, k, x.shape[0], _p(y))
    return y


def t16_gemv_parts(x_bf16: np.ndarray, qs: np.ndarray, d: np.ndarray, kp: int, ks: int) -> np.ndarray:
    """Persistent-step GEMV order: fp32 parts [kp, n] (x staged at S = 13 - e)."""
    xf = bf16_to_f32(np.ascontiguousarray(x_bf16, dtype=np.uint16)).astype(np.float32)
    n, k = qs.shape[0], qs.shape[1] * 2
    parts = np.empty((kp, n), np.float32)
    lib().orc_t16_gemv_parts(_p(np.ascontiguousarray(xf)), _p(np.ascontiguousarray(qs)),
                             _p(np.ascontiguousarray(d)), n, k, kp, ks, _p(parts))
    return parts


def q6k_dequantize(blocks: np.ndarray) -> np.ndarray:
    """Q6_K super-blocks uint8 [..., 210] -> fp32 [n_blocks * 256] (gguf's decode)."""
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1, 210)
    w = np.empty(b.shape[0] * 256, np.float32)
    lib().orc_q6k_dequantize(_p(b), b.shape[0], _p(w))
    return w


def q6k_gemv_parts(x_bf16: np.ndarray, blocks: np.ndarray, n: int, k: int, kp: int, ks: int) -> np.ndarray:
    """Persistent-step Q6_K GEMV order: fp32 parts [kp, n] for gguf Q6_K rows
    (uint8 [n, k / 256 * 210]) and bf16 x [k]."""
    xf = bf16_to_f32(np.ascontiguousarray(x_bf16, dtype=np.uint16)).astype(np.float32)
    parts = np.empty((kp, n), np.float32)
    lib().orc_q6k_gemv_parts(_p(np.ascontiguousarray(xf)), _p(np.ascontiguousarray(blocks, dtype=np.uint8)), n, k,
                             kp, ks, _p(parts))
    return parts


def parts_to_bf16(parts: np.ndarray) -> np.ndarray:
    parts = np.ascontiguousarray(parts, dtype=np.float32)
    kp, n = parts.shape
    y = np.empty(n, np.uint16)
    lib().orc_parts_to_bf16(_p(parts), kp, n, _p(y))
    return y


def t16_gemv(x_bf16: np.ndarray, qs: np.ndarray, d: np.ndarray, kp: int, ks: int) -> np.ndarray:
    return parts_to_bf16(t16_gemv_parts(x_bf16, qs, d, kp, ks))


# ----------------------------------------------------------------- elementwise
def add_rmsnorm(a, b, gamma, eps: float, want_res: bool = True):
    a = np.ascontiguousarray(a, dtype=np.uint16)
    h = a.shape[-1]
    bb = None if b is None else np.ascontiguousarray(b, dtype=np.uint16)
    g = np.ascontiguousarray(gamma, dtype=np.uint16)
    res = np.empty(h, np.uint16) if want_res else None
    y = np.empty(h, np.uint16)
    lib().orc_add_rmsnorm(_p(a), _p(bb), _p(g), h, eps, _p(res), _p(y))
    return res, y


def rope_neox(x_bf16: np.ndarray, cs_row: np.ndarray) -> np.ndarray:
    x = np.array(x_bf16, dtype=np.uint16, copy=True, order="C")
    nh, dim = x.shape
    lib().orc_rope_neox(_p(x), nh, dim, _p(np.ascontiguousarray(cs_row, dtype=np.uint16)))
    return x


def silu_mul(g, u) -> np.ndarray:
    g = np.ascontiguousarray(g, dtype=np.uint16)
    u = np.ascontiguousarray(u, dtype=np.uint16)
    out = np.empty_like(g)
    lib().orc_silu_mul(_p(g), _p(u), g.size, _p(out))
    return out


def exp(x: float) -> float:
    return lib().orc_exp(x)


def log(x: float) -> float:
    return lib().orc_log(x)


# ----------------------------------------------------------------- paged KV / attention
def slot_mapping(positions: np.ndarray, table: np.ndarray, block_size: int, max_tokens: int,
                 start: int = 0, end: int | None = None) -> np.ndarray:
    pos = np.ascontiguousarray(positions, dtype=np.int64)
    n = pos.size
    end = n if end is None else end
    out = np.empty(max_tokens, np.int64)
    lib().orc_slot_mapping(n, max_tokens, start, end, _p(pos), _p(np.ascontiguousarray(table, dtype=np.int32)),
                           block_size, _p(out))
    return out


def split_tokens(length: int, splits: int) -> int:
    return lib().orc_split_tokens(length, splits)


def attn_split(q, kc, vc, table, length: int, splits: int, scale: float, chunk_accs: int = 0, window: int = 0):
    """q bf16 [nq, D]; kc/vc bf16 [blocks, nkv, bs, D]; returns (part_o [S,nq,D], part_lse [S,nq]).
    ``chunk_accs`` > 0 selects the persistent-step order with that many consumer warps
    (scores over D / 16 lanes per token; each split cut into that many token ranges, each
    with its own softmax, merged by their maxima); ``window`` > 0: only the last
    ``window`` positions (Spark sliding layers)."""
    q = np.ascontiguousarray(q, dtype=np.uint16)
    kc = np.ascontiguousarray(kc, dtype=np.uint16)
    vc = np.ascontiguousarray(vc, dtype=np.uint16)
    nq, dim = q.shape
    _, nkv, bs, _ = kc.shape
    po = np.empty((splits, nq, dim), np.float32)
    pl = np.empty((splits, nq), np.float32)
    lib().orc_attn_split_x(_p(q), _p(kc), _p(vc), _p(np.ascontiguousarray(table, dtype=np.int32)), length, nq,
                           nkv, dim, bs, splits, scale, chunk_accs, window, _p(po), _p(pl))
    return po, pl


def attn_combine(part_o, part_lse, gate=None) -> np.ndarray:
    """``gate`` bf16 [nq] (Spark headwise output gate) or None."""
    po = np.ascontiguousarray(part_o, dtype=np.float32)
    pl = np.ascontiguousarray(part_lse, dtype=np.float32)
    splits, nq, dim = po.shape
    out = np.empty((nq, dim), np.uint16)
    g = None if gate is None else np.ascontiguousarray(gate, dtype=np.uint16)
    lib().orc_attn_combine_g(_p(po), _p(pl), splits, nq, dim, _p(g), _p(out))
    return out


def rope_partial(x_bf16: np.ndarray, rot: int, cs_row: np.ndarray) -> np.ndarray:
    """x bf16 [nh, D]; pairs (i, i + rot/2) rotated with a cos | sin row of rot entries."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16).copy()
    nh, dim = x.shape
    lib().orc_rope_partial(_p(x), nh, dim, rot, _p(np.ascontiguousarray(cs_row, dtype=np.uint16)))
    return x


def gelu_table() -> np.ndarray:
    """The reference's GELU table (integration/model.py:12-16): torch's exact-erf gelu of
    every bf16 input, kept for |x| in [2^-9, 128) -- inputs 0x3b00 + i, then 0xbb00 + i."""
    import torch
    bits = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    full = torch.nn.functional.gelu(bits, approximate="none")
    t = torch.cat((full[0x3B00:0x4300], full[0xBB00:0xC300])).contiguous()
    return t.view(torch.int16).numpy().view(np.uint16).copy()


def gelu_mul(g, u, table) -> np.ndarray:
    g = np.ascontiguousarray(g, dtype=np.uint16)
    u = np.ascontiguousarray(u, dtype=np.uint16)
    out = np.empty_like(g)
    lib().orc_gelu_mul(_p(g), _p(u), g.size, _p(np.ascontiguousarray(table, dtype=np.uint16)), _p(out))
    return out


def sigmoid_bf16(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.uint16)
    out = np.empty_like(x)
    lib().orc_sigmoid_bf16(_p(x), x.size, _p(out))
    return out


def argmax_bf16(logits) -> int:
    lg = np.ascontiguousarray(logits, dtype=np.uint16)
    return int(lib().orc_argmax_bf16(_p(lg), lg.size))


def set_threads(n: int) -> None:
    lib().orc_set_threads(n)


def get_threads() -> int:
    return lib().orc_get_threads()


# ----------------------------------------------------------------- whole model
class OracleModel:
    """Host copy of a synthetic Spark decoder for the C decode step.

    ``weights`` is a dict of numpy arrays with the keys produced by
    ``spark_b200.model.SyntheticWeights.to_numpy()``.
    """

    def __init__(self, cfg, weights: dict, num_blocks: int, splits: int, order: dict | None = None):
        """``order`` None: per-kernel evaluation order.  Persistent-step order:
        {"ks": (qkv, o, gate_up, down, head), "kp": (o, down), "chunk_accs": W}."""
        if splits <= 0:
            raise ValueError(f"splits must be positive, got {splits}")
        self.cfg = cfg
        self.w = weights
        self.splits = splits
        self.num_blocks = num_blocks
        L, nkv, bs, D = cfg.num_layers, cfg.num_kv_heads, cfg.block_size, cfg.head_dim
        self.kc = np.zeros((L, num_blocks, nkv, bs, D), np.uint16)
        self.vc = np.zeros_like(self.kc)
        self.dims = np.array([cfg.hidden_size, cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim,
                              cfg.intermediate_size, cfg.vocab_size, cfg.num_layers, cfg.block_size,
                              splits, cfg.max_position], dtype=np.int64)
        if order is None:
            ext = [0] * 9
        else:
            ext = [1, *order["ks"], *order["kp"], order["chunk_accs"]]
        self.dims = np.concatenate([self.dims, np.array(ext, dtype=np.int64)])
        self._keep = []
        mp = [weights["embed"], weights["final_norm"], weights["head_qs"], weights["head_d"], weights["cos_sin"]]
        self.model_ptrs = (ctypes.c_void_p * 5)(*[_p(a) for a in mp])
        lp = []
        for li in range(L):
            for key in ("in_norm", "post_norm", "qkv_qs", "qkv_d", "o_qs", "o_d", "gu_qs", "gu_d",
                        "down_qs", "down_d"):
                lp.append(_p(weights[f"layers.{li}.{key}"]))
        self.layer_ptrs = (ctypes.c_void_p * len(lp))(*lp)

    def layer(self, li: int, a: np.ndarray, b: np.ndarray, has_b: bool, table: np.ndarray, pos: int) -> None:
        """One decoder layer in place: a <- down projection, b <- residual (resmid)."""
        cfg = self.cfg
        kc, vc = self.kc[li], self.vc[li]
        lp = ctypes.cast(ctypes.byref(self.layer_ptrs, li * 10 * ctypes.sizeof(ctypes.c_void_p)),
                         ctypes.POINTER(ctypes.c_void_p))
        lib().orc_decode_layer(_p(self.dims), lp, _p(self.w["cos_sin"]), _p(kc), _p(vc),
                               _p(np.ascontiguousarray(table, dtype=np.int32)), pos, cfg.rms_norm_eps,
                               cfg.attn_scale, _p(a), _p(b), 1 if has_b else 0)

    def head(self, a: np.ndarray, b: np.ndarray) -> int:
        return int(lib().orc_decode_head(_p(self.dims), self.model_ptrs, _p(a), _p(b), self.cfg.rms_norm_eps, None))

    def step(self, table: np.ndarray, token: int, pos: int, want_logits: bool = False):
        cfg = self.cfg
        logits = np.empty(cfg.vocab_size, np.uint16) if want_logits else None
        table = np.ascontiguousarray(table, dtype=np.int32)
        tok = lib().orc_decode_step(_p(self.dims), self.model_ptrs, self.layer_ptrs, _p(self.kc), _p(self.vc),
                                    self.num_blocks, _p(table), token, pos, cfg.rms_norm_eps,
                                    cfg.attn_scale, _p(logits))
        return (int(tok), logits) if want_logits else int(tok)


class SparkOracleModel:
    """Host decoder of the Spark architecture in the persistent-step order.

    The same steps as ``orc_decode_layer`` / ``orc_decode_step`` (add + RMSNorm, T16
    GEMVs, RoPE, paged KV store, split attention and combine, MLP, head), with the Spark
    layer features of the reference (plugin/spark2_5.py:140-241): the gate rows after the
    qkv heads give bf16 sigmoid gates that multiply the combined attention heads
    (vector.py:81); full layers rotate ``rotary_dim`` dims with their theta, sliding
    layers the whole head with theirs and attend to the last ``sliding_window`` positions
    (attention.py:124-127); GELU * mul through the reference's table (linear.py:540-577);
    the LM head is the tied Q6_K embedding when ``weights`` has ``head_q6``.
    ``order``: the engine's persistent-step order ({"ks", "kp", "chunk_accs"})."""

    def __init__(self, cfg, weights: dict, num_blocks: int, splits: int, order: dict):
        self.cfg, self.w, self.splits, self.order = cfg, weights, splits, order
        L, nkv, bs, D = cfg.num_layers, cfg.num_kv_heads, cfg.block_size, cfg.head_dim
        self.kc = np.zeros((L, num_blocks, nkv, bs, D), np.uint16)
        self.vc = np.zeros_like(self.kc)
        self.gelu = gelu_table() if cfg.hidden_act == "gelu" else None

    def layer(self, li: int, a: np.ndarray, b: np.ndarray | None, table: np.ndarray, pos: int):
        """One decoder layer: returns (down projection, residual after attention)."""
        cfg, w, o = self.cfg, self.w, self.order
        p = f"layers.{li}."
        ks_qkv, ks_o, ks_gu, ks_down, _ = o["ks"]
        kp_o, kp_down = o["kp"]
        nq, nkv, D, bs, eps = cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim, cfg.block_size, cfg.rms_norm_eps
        nh = nq + 2 * nkv
        res, x = add_rmsnorm(a, b, w[p + "in_norm"], eps)
        y = t16_gemv(x, w[p + "qkv_qs"], w[p + "qkv_d"], 1, ks_qkv)
        qkv = y[:nh * D].reshape(nh, D)
        _, r = cfg.layer_rope(li)
        cs = w["cos_sin_sliding"] if cfg.is_sliding(li) else w["cos_sin"]
        rot = rope_partial(qkv[:nq + nkv], r, cs[pos])
        blk, off = int(table[pos // bs]), pos % bs
        self.kc[li, blk, :, off] = rot[nq:]
        self.vc[li, blk, :, off] = qkv[nq + nkv:]
        gate = sigmoid_bf16(y[nh * D:nh * D + nq]) if cfg.attn_gate else None
        po, pl = attn_split(rot[:nq], self.kc[li], self.vc[li], table, pos + 1, self.splits, cfg.attn_scale,
                            chunk_accs=o["chunk_accs"], window=cfg.layer_window(li))
        attn = attn_combine(po, pl, gate).reshape(-1)
        oproj = t16_gemv(attn, w[p + "o_qs"], w[p + "o_d"], kp_o, ks_o)
        resmid, x2 = add_rmsnorm(oproj, res, w[p + "post_norm"], eps)
        gu = t16_gemv(x2, w[p + "gu_qs"], w[p + "gu_d"], 1, ks_gu)
        i = cfg.intermediate_size
        mid = gelu_mul(gu[:i], gu[i:], self.gelu) if self.gelu is not None else silu_mul(gu[:i], gu[i:])
        return t16_gemv(mid, w[p + "down_qs"], w[p + "down_d"], kp_down, ks_down), resmid

    def head(self, a: np.ndarray, b: np.ndarray):
        cfg, w = self.cfg, self.w
        _, x = add_rmsnorm(a, b, w["final_norm"], cfg.rms_norm_eps, want_res=False)
        ks = self.order["ks"][4]
        if "head_q6" in w:
            logits = parts_to_bf16(q6k_gemv_parts(x, w["head_q6"], cfg.vocab_size, cfg.hidden_size, 1, ks))
        else:
            logits = t16_gemv(x, w["head_qs"], w["head_d"], 1, ks)
        return argmax_bf16(logits), logits

    def step(self, table: np.ndarray, token: int, pos: int, want_logits: bool = False):
        table = np.ascontiguousarray(table, dtype=np.int32)
        a, b = self.w["embed"][token].copy(), None
        for li in range(self.cfg.num_layers):
            a, b = self.layer(li, a, b, table, pos)
        tok, logits = self.head(a, b)
        return (tok, logits) if want_logits else tok
