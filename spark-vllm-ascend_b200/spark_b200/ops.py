"""Torch-facing operators over the C ABI, plus ``torch.ops.spark_b200.*`` registrations.

Two layers:

* ``*_out`` functions take caller-owned output tensors, allocate nothing and
  launch on the current CUDA stream -- this is what the decode engine captures
  into a CUDA graph.
* ``torch.ops.spark_b200.<name>`` custom ops (``torch.library.custom_op``) that
  allocate their outputs; they are what the vLLM quantized-linear method and
  attention backend call.  Each has a fake (meta) implementation so that
  torch.compile can trace through it.

Argument checks mirror the reference's native op (native/head/extension.cpp:8-10):
device, dtype, layout and size are validated before the launch, and a bad call
raises instead of reaching the kernel.
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import call

BF16 = torch.bfloat16


def _p(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _cuda(t: torch.Tensor, name: str, dtype: torch.dtype | None = None) -> None:
    _check(t.is_cuda, f"{name} must be a CUDA tensor")
    _check(t.is_contiguous(), f"{name} must be contiguous")
    if dtype is not None:
        _check(t.dtype == dtype, f"{name} must be {dtype}, got {t.dtype}")


def _q4(qs: torch.Tensor, d: torch.Tensor) -> tuple[int, int]:
    _cuda(qs, "qs", torch.uint8)
    _cuda(d, "d")
    _check(d.dtype in (torch.float16, torch.uint16, torch.int16), "d must hold fp16 scales")
    _check(qs.dim() == 2 and d.dim() == 2, "qs / d must be 2-D")
    n, k = qs.shape[0], qs.shape[1] * 2
    _check(d.shape == (n, k // 32), f"d must be [{n}, {k // 32}], got {tuple(d.shape)}")
    return n, k


# ---------------------------------------------------------------- Q4_0 format
def q4_quantize(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 [rows, k] on the GPU -> (qs uint8 [rows, k/2], d fp16 [rows, k/32]); gguf Q4_0."""
    _cuda(w, "w", torch.float32)
    rows, k = w.shape
    qs = torch.empty((rows, k // 2), dtype=torch.uint8, device=w.device)
    d = torch.empty((rows, k // 32), dtype=torch.float16, device=w.device)
    call("spark_q4_quantize", _p(w), rows, k, _p(qs), _p(d), _stream())
    return qs, d


def q4_split_gguf(blocks: torch.Tensor, rows: int, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    _cuda(blocks, "blocks", torch.uint8)
    _check(blocks.numel() == rows * (k // 32) * 18, "blocks size mismatch")
    qs = torch.empty((rows, k // 2), dtype=torch.uint8, device=blocks.device)
    d = torch.empty((rows, k // 32), dtype=torch.float16, device=blocks.device)
    call("spark_q4_split_gguf", _p(blocks), rows, k, _p(qs), _p(d), _stream())
    return qs, d


def q4_dequantize(qs: torch.Tensor, d: torch.Tensor) -> torch.Tensor:
    n, k = _q4(qs, d)
    w = torch.empty((n, k), dtype=BF16, device=qs.device)
    call("spark_q4_dequantize_bf16", _p(qs), _p(d), n, k, _p(w), _stream())
    return w


def q4_gemm(x: torch.Tensor, qs: torch.Tensor, d: torch.Tensor, error: torch.Tensor,
            wait_ns: int = -1) -> torch.Tensor:
    """Prefill GEMM on the tensor cores: x bf16 [T, K] times the Q4_0 weight [N, K]
    (dequantized in shared memory) -> bf16 [T, N].  K % 256 == 0.  ``error`` (int32 [1],
    required, on the device) becomes nonzero if a wait inside the kernel ran out, and y
    is then not valid: the caller owns the status word and must read it.  ``wait_ns``
    bounds each wait (-1: the kernel's 0.5 s; 0: give up at once, for tests)."""
    n, k = _q4(qs, d)
    _cuda(x, "x", BF16)
    _cuda(error, "error", torch.int32)
    _check(error.numel() >= 1, "error must hold one int32")
    x2 = x.reshape(-1, k)
    _check(x2.is_contiguous(), "x must be contiguous")
    t = x2.shape[0]
    y = torch.empty((t, n), dtype=BF16, device=x.device)
    call("spark_q4_gemm_tc", _p(x2), _p(qs), _p(d), _p(y), t, n, k, _p(error), int(wait_ns), _stream())
    return y


# ---------------------------------------------------------------- GEMV family
def q4_gemv_out(x: torch.Tensor, qs: torch.Tensor, d: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    n, k = _q4(qs, d)
    _cuda(x, "x", BF16)
    _cuda(y, "y", BF16)
    x2 = x.reshape(-1, k)
    batch = x2.shape[0]
    _check(1 <= batch <= 8, "batch must be in 1..8")
    _check(y.numel() == batch * n, "y has the wrong size")
    call("spark_q4_gemv", _p(x2), _p(qs), _p(d), _p(y), n, k, batch, _stream())
    return y


def q4_gemv(x: torch.Tensor, qs: torch.Tensor, d: torch.Tensor) -> torch.Tensor:
    n, k = _q4(qs, d)
    y = torch.empty((*x.shape[:-1], n), dtype=BF16, device=x.device)
    return q4_gemv_out(x, qs, d, y)


def rmsnorm_q4_gemv_out(a, b, gamma, eps, qs, d, y, res_out=None):
    n, k = _q4(qs, d)
    for t, nm in ((a, "a"), (gamma, "gamma"), (y, "y")):
        _cuda(t, nm, BF16)
    _check(a.numel() == k and gamma.numel() == k and y.numel() == n, "size mismatch")
    if b is not None:
        _cuda(b, "b", BF16)
    call("spark_rmsnorm_q4_gemv", _p(a), _p(b), _p(gamma), float(eps), _p(res_out), _p(qs), _p(d), _p(y), n, k,
         _stream())
    return y


def rmsnorm_gate_up_silu_out(a, b, gamma, eps, qs, d, mid, res_out=None):
    n, k = _q4(qs, d)
    for t, nm in ((a, "a"), (gamma, "gamma"), (mid, "mid")):
        _cuda(t, nm, BF16)
    _check(a.numel() == k and mid.numel() == n // 2, "size mismatch")
    call("spark_rmsnorm_gate_up_silu", _p(a), _p(b), _p(gamma), float(eps), _p(res_out), _p(qs), _p(d), _p(mid), n,
         k, _stream())
    return mid


def qkv_rope_kvstore_out(a, b, gamma, eps, qs, d, nq, nkv, head_dim, cos_sin, pos, block_table, slot_mapping,
                         block_size, k_cache, v_cache, q_out, res_out=None, embed=None, token=None):
    n, k = _q4(qs, d)
    _check(n == (nq + 2 * nkv) * head_dim, "qkv weight rows must be (nq + 2 nkv) * head_dim")
    _cuda(gamma, "gamma", BF16)
    _cuda(cos_sin, "cos_sin", BF16)
    _cuda(k_cache, "k_cache", BF16)
    _cuda(v_cache, "v_cache", BF16)
    _cuda(q_out, "q_out", BF16)
    _cuda(pos, "pos", torch.int64)
    call("spark_qkv_rope_kvstore", _p(a), _p(b), _p(embed), _p(token), _p(gamma), float(eps), _p(res_out), _p(qs),
         _p(d), k, nq, nkv, head_dim, _p(cos_sin), _p(pos), _p(block_table), _p(slot_mapping), block_size,
         _p(k_cache), _p(v_cache), _p(q_out), _stream())
    return q_out


def head_argmax_out(a, b, gamma, eps, qs, d, logits, key):
    n, k = _q4(qs, d)
    _cuda(logits, "logits", BF16)
    _check(key.dtype in (torch.int64, torch.uint64) and key.is_cuda, "key must be a CUDA int64 tensor")
    call("spark_rmsnorm_q4_head_argmax", _p(a), _p(b), _p(gamma), float(eps), _p(qs), _p(d), _p(logits), n, k,
         _p(key), _stream())
    return logits


def decode_finalize(key, token_out, token_log=None, step=None, pos=None):
    call("spark_decode_finalize", _p(key), _p(token_out), _p(token_log), _p(step), _p(pos), _stream())


# ---------------------------------------------------------------- attention
def attn_splitkv_out(q, k_cache, v_cache, block_table, splits, max_split_tokens, scale, part_o, part_lse,
                     pos=None, seq_len=None, error=None):
    _cuda(q, "q", BF16)
    nq, head_dim = q.shape[-2], q.shape[-1]
    _cuda(k_cache, "k_cache", BF16)
    _cuda(v_cache, "v_cache", BF16)
    _check(k_cache.dim() == 4 and k_cache.shape == v_cache.shape, "caches must be [blocks, nkv, block_size, D]")
    nkv, block_size = k_cache.shape[1], k_cache.shape[2]
    _check(k_cache.shape[3] == head_dim, "head_dim mismatch")
    _cuda(block_table, "block_table", torch.int32)
    _check(part_o.shape == (splits, nq, head_dim) and part_lse.shape == (splits, nq), "partials shape")
    _check((pos is None) != (seq_len is None), "give exactly one of pos / seq_len")
    if pos is not None:
        _cuda(pos, "pos", torch.int64)
    if seq_len is not None:
        _cuda(seq_len, "seq_len", torch.int32)
    call("spark_attn_splitkv", _p(q), _p(k_cache), _p(v_cache), _p(block_table), _p(pos), _p(seq_len), nq, nkv,
         head_dim, block_size, splits, max_split_tokens, float(scale), _p(part_o), _p(part_lse), _p(error), _stream())


def attn_decode_out(q, k_cache, v_cache, block_table, splits, max_split_tokens, scale, part_o, part_lse, counters,
                    out, pos=None, seq_len=None, error=None):
    """Split-KV attention with the fused LSE combine (counters: int32 [nkv], zero)."""
    _cuda(q, "q", BF16)
    nq, head_dim = q.shape[-2], q.shape[-1]
    _check(k_cache.dim() == 4 and k_cache.shape == v_cache.shape, "caches must be [blocks, nkv, block_size, D]")
    nkv, block_size = k_cache.shape[1], k_cache.shape[2]
    _cuda(counters, "counters", torch.int32)
    _cuda(out, "out", BF16)
    _check((pos is None) != (seq_len is None), "give exactly one of pos / seq_len")
    call("spark_attn_decode", _p(q), _p(k_cache), _p(v_cache), _p(block_table), _p(pos), _p(seq_len), nq, nkv,
         head_dim, block_size, splits, max_split_tokens, float(scale), _p(part_o), _p(part_lse), _p(counters),
         _p(out), _p(error), _stream())
    return out


def attn_combine_out(part_o, part_lse, out):
    splits, nq, head_dim = part_o.shape
    _cuda(part_o, "part_o", torch.float32)
    _cuda(part_lse, "part_lse", torch.float32)
    _cuda(out, "out", BF16)
    call("spark_attn_combine", _p(part_o), _p(part_lse), splits, nq, head_dim, _p(out), _stream())
    return out


# ---------------------------------------------------------------- elementwise
def add_rmsnorm_out(a, b, gamma, eps, y, res_out=None):
    _cuda(a, "a", BF16)
    _cuda(gamma, "gamma", BF16)
    h = a.numel()
    call("spark_add_rmsnorm", _p(a), _p(b), _p(gamma), float(eps), h, _p(res_out), _p(y), _stream())
    return y


def silu_mul_out(g, u, out):
    _cuda(g, "g", BF16)
    _cuda(u, "u", BF16)
    call("spark_silu_mul", _p(g), _p(u), g.numel(), _p(out), _stream())
    return out


def rope_neox_(x, cos_sin, pos):
    _cuda(x, "x", BF16)
    nh, dim = x.shape[-2], x.shape[-1]
    call("spark_rope_neox", _p(x), nh, dim, _p(cos_sin), _p(pos), _stream())
    return x


def add_rmsnorm_rows(a: torch.Tensor, b: torch.Tensor | None, gamma: torch.Tensor, eps: float):
    """Prefill rows: a / b bf16 [n, h] -> (bf16(a + b), bf16 RMSNorm(a + b) * gamma)."""
    _cuda(a, "a", BF16)
    _cuda(gamma, "gamma", BF16)
    n, h = a.shape
    a = a.contiguous()
    b = None if b is None else b.contiguous()
    res, y = torch.empty_like(a), torch.empty_like(a)
    call("spark_add_rmsnorm_rows", _p(a), _p(b), _p(gamma), float(eps), n, h, _p(res), _p(y), _stream())
    return res, y


def rope_rows_(x: torch.Tensor, nh: int, head_dim: int, rotary_dim: int, cos_sin: torch.Tensor, pos0: int):
    """In-place RoPE of the first ``nh`` heads of each row of x (bf16 [n, >= nh * head_dim],
    rows contiguous), row r at position pos0 + r."""
    _cuda(x, "x", BF16)
    _check(x.dim() == 2 and x.stride(1) == 1, "x must be [rows, cols] with contiguous rows")
    call("spark_rope_neox_rows", _p(x), x.stride(0), x.shape[0], nh, head_dim, rotary_dim, _p(cos_sin), pos0,
         _stream())
    return x


def act_mul_rows(gu: torch.Tensor, gelu_table: torch.Tensor | None = None) -> torch.Tensor:
    """gu bf16 [n, 2 I] (gate | up) -> bf16 [n, I] = act(gate) * up (SiLU, or GELU by the
    table of ``step.gelu_table``), the decode epilogues' arithmetic."""
    _cuda(gu, "gu", BF16)
    n, i2 = gu.shape
    gu = gu.contiguous()
    out = torch.empty((n, i2 // 2), dtype=BF16, device=gu.device)
    call("spark_act_mul_rows", _p(gu), n, i2 // 2, _p(gelu_table), _p(out), _stream())
    return out


def slot_mapping_out(num_tokens, query_start, positions, block_table, block_size, out):
    _cuda(out, "out", torch.int64)
    call("spark_slot_mapping", num_tokens, out.numel(), _p(query_start), _p(positions), _p(block_table), block_size,
         _p(out), _stream())
    return out


def kv_store_(k: torch.Tensor, v: torch.Tensor, slot_mapping: torch.Tensor, k_cache: torch.Tensor,
              v_cache: torch.Tensor) -> None:
    """Scatter k / v [tokens, nkv, D] into the paged caches [blocks, nkv, bs, D] at
    slot_mapping (int64; negative slots skipped)."""
    _cuda(k, "k", BF16)
    _cuda(v, "v", BF16)
    _cuda(slot_mapping, "slot_mapping", torch.int64)
    _cuda(k_cache, "k_cache", BF16)
    _cuda(v_cache, "v_cache", BF16)
    t, nkv, d = k.shape
    _check(k_cache.dim() == 4 and k_cache.shape[1] == nkv and k_cache.shape[3] == d, "k_cache shape")
    call("spark_kv_store", _p(k.contiguous()), _p(v.contiguous()), _p(slot_mapping.contiguous()), t, nkv, d,
         k_cache.shape[2], _p(k_cache), _p(v_cache), _stream())


def set_pdl(enabled: bool) -> None:
    call("spark_set_pdl", 1 if enabled else 0)


def set_gemv_ring(enabled: bool) -> None:
    """Choose the weight-ring GEMV (default) or the register-direct GEMV for K % 512 == 0."""
    call("spark_set_gemv_ring", 1 if enabled else 0)


def read_device_error(reset: bool = True) -> int:
    """Synchronously read (and optionally clear) the library's device error word."""
    v = ctypes.c_int(0)
    call("spark_read_device_error", ctypes.byref(v), 1 if reset else 0)
    return int(v.value)


# ---------------------------------------------------------------- torch.library custom ops
@torch.library.custom_op("spark_b200::q4_gemv", mutates_args=())
def _op_q4_gemv(x: torch.Tensor, qs: torch.Tensor, d: torch.Tensor) -> torch.Tensor:
    return q4_gemv(x.contiguous(), qs, d)


@_op_q4_gemv.register_fake
def _(x, qs, d):
    return x.new_empty((*x.shape[:-1], qs.shape[0]))


@torch.library.custom_op("spark_b200::rmsnorm_q4_gemv", mutates_args=())
def _op_rmsnorm_q4_gemv(a: torch.Tensor, b: torch.Tensor | None, gamma: torch.Tensor, eps: float,
                        qs: torch.Tensor, d: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    y = a.new_empty((qs.shape[0],))
    res = torch.empty_like(a)
    rmsnorm_q4_gemv_out(a.contiguous(), None if b is None else b.contiguous(), gamma, eps, qs, d, y, res)
    return y, res


@_op_rmsnorm_q4_gemv.register_fake
def _(a, b, gamma, eps, qs, d):
    return a.new_empty((qs.shape[0],)), torch.empty_like(a)


@torch.library.custom_op("spark_b200::rmsnorm_gate_up_silu", mutates_args=())
def _op_gate_up(a: torch.Tensor, b: torch.Tensor | None, gamma: torch.Tensor, eps: float, qs: torch.Tensor,
                d: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    mid = a.new_empty((qs.shape[0] // 2,))
    res = torch.empty_like(a)
    rmsnorm_gate_up_silu_out(a.contiguous(), None if b is None else b.contiguous(), gamma, eps, qs, d, mid, res)
    return mid, res


@_op_gate_up.register_fake
def _(a, b, gamma, eps, qs, d):
    return a.new_empty((qs.shape[0] // 2,)), torch.empty_like(a)


@torch.library.custom_op("spark_b200::qkv_rope_kvstore", mutates_args=("k_cache", "v_cache"))
def _op_qkv(a: torch.Tensor, b: torch.Tensor | None, gamma: torch.Tensor, eps: float, qs: torch.Tensor,
            d: torch.Tensor, nq: int, nkv: int, head_dim: int, cos_sin: torch.Tensor, pos: torch.Tensor,
            slot_mapping: torch.Tensor, block_size: int, k_cache: torch.Tensor,
            v_cache: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    q = a.new_empty((nq, head_dim))
    res = torch.empty_like(a)
    qkv_rope_kvstore_out(a.contiguous(), None if b is None else b.contiguous(), gamma, eps, qs, d, nq, nkv,
                         head_dim, cos_sin, pos, None, slot_mapping, block_size, k_cache, v_cache, q, res)
    return q, res


@_op_qkv.register_fake
def _(a, b, gamma, eps, qs, d, nq, nkv, head_dim, cos_sin, pos, slot_mapping, block_size, k_cache, v_cache):
    return a.new_empty((nq, head_dim)), torch.empty_like(a)


@torch.library.custom_op("spark_b200::attn_decode", mutates_args=())
def _op_attn(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor,
             seq_len: torch.Tensor, splits: int, max_split_tokens: int, scale: float) -> torch.Tensor:
    nq, dim = q.shape[-2], q.shape[-1]
    part_o = torch.empty((splits, nq, dim), dtype=torch.float32, device=q.device)
    part_lse = torch.empty((splits, nq), dtype=torch.float32, device=q.device)
    attn_splitkv_out(q.contiguous(), k_cache, v_cache, block_table, splits, max_split_tokens, scale, part_o, part_lse,
                     seq_len=seq_len)
    out = q.new_empty((nq, dim))
    attn_combine_out(part_o, part_lse, out)
    return out


@_op_attn.register_fake
def _(q, k_cache, v_cache, block_table, seq_len, splits, max_split_tokens, scale):
    return q.new_empty((q.shape[-2], q.shape[-1]))


@torch.library.custom_op("spark_b200::add_rmsnorm", mutates_args=())
def _op_add_rmsnorm(a: torch.Tensor, b: torch.Tensor | None, gamma: torch.Tensor,
                    eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    y = torch.empty_like(a)
    res = torch.empty_like(a)
    add_rmsnorm_out(a.contiguous(), None if b is None else b.contiguous(), gamma, eps, y, res)
    return y, res


@_op_add_rmsnorm.register_fake
def _(a, b, gamma, eps):
    return torch.empty_like(a), torch.empty_like(a)


@torch.library.custom_op("spark_b200::silu_mul", mutates_args=())
def _op_silu_mul(gu: torch.Tensor) -> torch.Tensor:
    half = gu.shape[-1] // 2
    g = gu[..., :half].contiguous()
    u = gu[..., half:].contiguous()
    out = torch.empty_like(g)
    silu_mul_out(g, u, out)
    return out


@_op_silu_mul.register_fake
def _(gu):
    return gu.new_empty((*gu.shape[:-1], gu.shape[-1] // 2))


def q6k_dequantize(blocks: torch.Tensor) -> torch.Tensor:
    """gguf Q6_K super-blocks (uint8 [..., 210] on the device) -> fp32 weights, the decode
    of gguf 0.19.0 (``spark_q6k_dequantize``)."""
    b = blocks.contiguous()
    if b.dtype != torch.uint8 or b.numel() % 210:
        raise ValueError("Q6_K blocks are uint8 rows of 210-byte super-blocks")
    nb = b.numel() // 210
    out = torch.empty(nb * 256, dtype=torch.float32, device=b.device)
    call("spark_q6k_dequantize", _p(b), nb, _p(out), _stream())
    return out
