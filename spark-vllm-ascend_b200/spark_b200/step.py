"""Persistent decode step: T16 weight packing and stage programs for ``spark_step_run``.

A decode step of the synthetic model is ONE cooperative kernel launch running a
program of stages (include/spark_b200.h, ``SparkStage``).  Per layer:

  qkv      GEMV, RMSNorm(a + b) prologue, RoPE + paged KV store epilogue
  attn     split-KV attention over the paged cache, last split of a head combines
  o_proj   GEMV, K split in ``kp_o`` parts -> fp32 parts
  gate_up  GEMV, RMSNorm(sum(o parts) + res) prologue, SiLU * mul epilogue
  down     GEMV, K split in ``kp_down`` parts -> fp32 parts (next layer's a)

then the LM head (RMSNorm prologue, argmax epilogue).  The last CTA of the launch
turns the argmax key into the next token and advances the position.
"""
from __future__ import annotations

import ctypes
import math

import torch

from ._lib import SparkStage, SparkStepIO, call, lib

STAGE_GEMV, STAGE_ATTN, STAGE_GEMV_Q6 = 0, 1, 2
PRO_BF16, PRO_PARTS, PRO_ATTN, PRO_PARTS_TAGGED = 0, 1, 2, 3
XCHG_LOCAL, XCHG_COUNTED, XCHG_TAGGED = 0, 1, 2
EPI_BF16, EPI_PARTS, EPI_ROPE_KV, EPI_SILU_MUL, EPI_ARGMAX, EPI_GELU_MUL = range(6)
ROWS_PLAIN, ROWS_PAIR_HALF, ROWS_GATE_UP = range(3)

MAX_SLICES = 4  # slices per GEMV unit the kernel supports
MAX_PARTS = 8  # fp32 parts a PARTS prologue sums (K parts x tensor-parallel ranks)
CHUNK_ACCS = 11  # consumer warps of the kernel = attention PV chunk accumulators
MAX_SPLIT_TOKENS = 1344
MAX_SPLITS = 127  # splits per kv head the attention stage's combine holds (kMaxCombineSplits)
TRACE_SLOTS = 24  # trace stamps per CTA and stage (kTraceSlots of the kernel)


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def num_ctas() -> int:
    return int(lib().spark_step_num_ctas())


def ring_bytes() -> int:
    return int(lib().spark_step_ring_bytes())


def t16_bytes(n: int, k: int, kp: int) -> int:
    return n * k * 9 // 16


def q4_pack_t16(qs: torch.Tensor, d: torch.Tensor, kp: int = 1, rowmap: int = ROWS_PLAIN,
                head_dim: int = 0, rotary_dim: int = 0) -> torch.Tensor:
    """Re-lay Q4_0 planes (qs uint8 [n, k/2], d fp16-bits [n, k/32]) as T16 units.
    ``ROWS_PAIR_HALF``: ``rotary_dim`` (Spark partial RoPE, 0 = head_dim) and rows past
    the last whole head (the Spark gate rows) as the qkv epilogue expects them."""
    n, k = qs.shape[0], qs.shape[1] * 2
    out = torch.empty(t16_bytes(n, k, kp), dtype=torch.uint8, device=qs.device)
    aux = head_dim | (rotary_dim << 16) if rowmap == ROWS_PAIR_HALF else head_dim
    call("spark_q4_pack_t16", _p(qs.contiguous()), _p(d.contiguous()), n, k, kp, rowmap, aux, _p(out), _stream())
    return out


def gelu_table(device) -> torch.Tensor:
    """The table of ``EPI_GELU_MUL``, bf16 [4096]: torch's exact-erf gelu of the bf16
    inputs 0x3b00 + i and 0xbb00 + i (|x| in [2^-9, 128)), built as the reference builds
    its activation table (integration/model.py:12-16); the kernel covers the rest of the
    range in closed form."""
    bits = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    full = torch.nn.functional.gelu(bits, approximate="none")
    return torch.cat((full[0x3B00:0x4300], full[0xBB00:0xC300])).contiguous().to(device)


def t6_bytes(n: int, k: int) -> int:
    return n * k * 105 // 128


def q6k_pack_t6(blocks: torch.Tensor, n: int, k: int, kp: int = 1) -> torch.Tensor:
    """Re-lay gguf Q6_K rows (uint8 [n, k / 256 * 210], on the device) as T6 units."""
    if blocks.dtype != torch.uint8 or blocks.numel() != n * (k // 256) * 210:
        raise ValueError("blocks must be uint8 gguf Q6_K rows [n, k / 256 * 210]")
    out = torch.empty(t6_bytes(n, k), dtype=torch.uint8, device=blocks.device)
    call("spark_q6k_pack_t6", _p(blocks.contiguous()), n, k, kp, _p(out), _stream())
    return out


def pick_ks(n: int, k: int, kp: int, want: int, ncta: int) -> int:
    """Largest slice count <= want (and <= MAX_SLICES) that divides the unit's
    64-column tiles."""
    tiles = (k // kp) // 64
    for ks in range(min(want, tiles, MAX_SLICES), 0, -1):
        if tiles % ks == 0:
            return ks
    raise ValueError(f"no slice count fits n={n} k={k} kp={kp}")


class StepProgram:
    """An ordered list of stages, its device copy, and the launch state.

    ``batch`` B > 1: a small-batch program (B in 2, 4, 8): every stage decodes B
    sequences, its buffers holding B copies of their one-sequence layout, sequence-major;
    ``bt_stride`` = entries per sequence row of the int32 [B][bt_stride] block table."""

    def __init__(self, device, ncta: int | None = None, batch: int = 1, bt_stride: int = 0):
        if batch not in (1, 2, 4, 8):
            raise ValueError(f"batch {batch}: the step kernel decodes 1, 2, 4 or 8 sequences")
        self.batch = batch
        self.bt_stride = bt_stride
        self.device = torch.device(device)
        self.ncta = ncta or num_ctas()
        self.stages: list[SparkStage] = []
        self.keep: list = []
        self._units = 0
        self.host = None
        self.dev = None
        self.counters = None

    # -- stage builders (return the stage index)
    def gemv(self, w: torch.Tensor, n: int, k: int, *, kp: int = 1, ks: int = 1, a=None, a_parts: int = 0,
             embed=None, token=None, b=None, gamma=None, eps: float = 0.0, res_out=None, epi: int = EPI_BF16,
             rowmap: int = ROWS_PLAIN, out=None, wait: int = -1, head_dim: int = 0, key=None, rope=None,
             xchg: int = 0, row0: int = 0, q6: bool = False, rotary_dim: int = 0, gate=None,
             table=None, attn_splits: int = 0, tagged: bool = False) -> int:
        """``xchg``: tensor-parallel exchange stage: XCHG_COUNTED (parts / argmax key
        written to every rank's window, completion counted on every rank) or XCHG_TAGGED
        (parts as tagged 64-bit words, not counted); ``tagged``: ``a`` holds tagged parts
        (``PRO_PARTS_TAGGED``, read once their tags are this launch's); ``row0``: global index of row 0
        for the argmax (vocab shard start); ``q6``: ``w`` holds Q6_K weights in the T6 layout
        (``q6k_pack_t6``); slices then count 32-weight tiles.  Spark layer features:
        ``rotary_dim`` (partial RoPE) and ``gate`` (bf16 [nq], computed from the gate rows
        after the heads) for ``EPI_ROPE_KV``; ``table`` (``gelu_table()``) for
        ``EPI_GELU_MUL``.  ``attn_splits`` > 0: an o_proj fused behind the attention stage
        added just before (``PRO_ATTN``: kp = its kv heads, input staged by it in shared
        memory, units assigned by head group; ``wait`` must be -1)."""
        s = SparkStage()
        s.kind, s.epi, s.rowmap = (STAGE_GEMV_Q6 if q6 else STAGE_GEMV), epi, rowmap
        s.pro = PRO_ATTN if attn_splits else ((PRO_PARTS_TAGGED if tagged else PRO_PARTS) if a_parts else PRO_BF16)
        s.splits = attn_splits
        s.n, s.k, s.kp, s.ks = n, k, kp, ks
        s.units = n // 16 * kp
        s.rot = self._units % self.ncta
        self._units += s.units
        s.wait = wait
        s.norm = 1 if gamma is not None else 0
        s.a_parts = a_parts
        s.eps = eps
        s.inv_k = float(torch.tensor(1.0 / k, dtype=torch.float32))
        s.head_dim = head_dim
        s.xchg, s.row0 = int(xchg), row0
        s.rotary_dim, s.gate, s.table = rotary_dim, _p(gate), _p(table)
        s.w, s.a, s.b, s.embed, s.token = _p(w), _p(a), _p(b), _p(embed), _p(token)
        s.gamma, s.res_out, s.out, s.key = _p(gamma), _p(res_out), _p(out), _p(key)
        if rope is not None:
            s.cos_sin, s.pos, s.block_table = _p(rope["cos_sin"]), _p(rope["pos"]), _p(rope["block_table"])
            s.k_cache, s.v_cache, s.q, s.kv_new = (_p(rope["k_cache"]), _p(rope["v_cache"]), _p(rope["q"]),
                                                   _p(rope["kv_new"]))
            s.block_size, s.nq, s.nkv = rope["block_size"], rope["nq"], rope["nkv"]
        self.keep.extend([w, a, b, embed, token, gamma, res_out, out, key, rope, gate, table])
        return self._add(s)

    def _add(self, s: SparkStage) -> int:
        if self.batch > 1:
            s.batch, s.bt_stride = self.batch, self.bt_stride
        self.stages.append(s)
        return len(self.stages) - 1

    def attention(self, *, q, k_cache, v_cache, kv_new, block_table, pos, splits: int, max_split_tokens: int,
                  scale: float, part_o, part_lse, head_counters, attn_out, nq: int, nkv: int, head_dim: int,
                  block_size: int, wait: int = -1, window: int = 0, gate=None) -> int:
        """Spark layer features: ``window`` > 0 attends to the last ``window`` positions
        (sliding layers); ``gate`` bf16 [nq] multiplies each head's output; head_dim 256."""
        s = SparkStage()
        s.kind = STAGE_ATTN
        s.wait = wait
        s.nq, s.nkv, s.head_dim, s.block_size = nq, nkv, head_dim, block_size
        s.splits, s.max_split_tokens, s.scale = splits, max_split_tokens, scale
        s.q, s.k_cache, s.v_cache, s.kv_new = _p(q), _p(k_cache), _p(v_cache), _p(kv_new)
        s.block_table, s.pos = _p(block_table), _p(pos)
        s.part_o, s.part_lse, s.head_counters, s.attn_out = _p(part_o), _p(part_lse), _p(head_counters), _p(attn_out)
        s.window, s.gate = window, _p(gate)
        self.keep.extend([q, k_cache, v_cache, kv_new, block_table, pos, part_o, part_lse, head_counters, attn_out,
                          gate])
        return self._add(s)

    # -- device copy
    def finalize(self, counters: torch.Tensor | None = None) -> "StepProgram":
        """``counters``: int32 [stages + 3] to use (tensor parallel: inside the exchange
        window), else allocated here."""
        n = len(self.stages)
        self.host = (SparkStage * n)(*self.stages)
        raw = torch.frombuffer(bytearray(bytes(self.host)), dtype=torch.uint8)
        self.dev = raw.to(self.device)
        if counters is not None:
            if counters.dtype != torch.int32 or counters.numel() < n + 3:
                raise ValueError(f"counters must be int32 with at least {n + 3} entries")
            self.counters = counters
        else:
            self.counters = torch.zeros(n + 3, dtype=torch.int32, device=self.device)
        return self

    def reset_counters(self) -> None:
        self.counters.zero_()

    def io(self, *, error=None, key=None, token_out=None, token_log=None, step=None, pos=None,
           trace=None, window=None) -> SparkStepIO:
        """``window``: the rank's connected ``tp.ExchangeWindow`` (tensor parallel)."""
        io = SparkStepIO()
        io.counters, io.error, io.key = _p(self.counters), _p(error), _p(key)
        io.token_out, io.token_log, io.step, io.pos = _p(token_out), _p(token_log), _p(step), _p(pos)
        io.trace = _p(trace)
        if window is not None:
            io.peer_windows, io.window = _p(window.peer_table), ctypes.c_void_p(window.ptr)
            io.window_bytes, io.tp_size, io.tp_rank = window.nbytes, window.size, window.rank
        else:
            io.tp_size, io.tp_rank = 1, 0
        return io

    def trace_buffer(self) -> torch.Tensor:
        """uint64 [ctas, stages, TRACE_SLOTS] for ``io(trace=...)``."""
        return torch.zeros((self.ncta, len(self.stages), TRACE_SLOTS), dtype=torch.int64, device=self.device)

    def launch(self, io: SparkStepIO, stream=None) -> None:
        if self.host is None:
            self.finalize()
        st = stream if stream is not None else _stream()
        dev = _p(self.dev) if len(self.stages) > 1 else None
        call("spark_step_run", ctypes.cast(self.host, ctypes.c_void_p), dev, len(self.stages),
             ctypes.byref(io), st)


def t16_gemv(x: torch.Tensor, w: torch.Tensor, n: int, k: int, kp: int = 1, ks: int = 1, parts: bool = False,
             **kw) -> torch.Tensor:
    """One T16 GEMV stage as its own launch (tests, kernel timing): bf16 out [n], or the
    fp32 parts [kp, n] when ``parts``."""
    dev = x.device
    if parts:
        out = torch.empty((kp, n), dtype=torch.float32, device=dev)
        epi = EPI_PARTS
    else:
        out = torch.empty(n, dtype=torch.bfloat16, device=dev)
        epi = EPI_BF16
    prog = StepProgram(dev)
    a_parts = kw.pop("a_parts", 0)
    prog.gemv(w, n, k, kp=kp, ks=ks, a=x, a_parts=a_parts, epi=epi, out=out, **kw)
    prog.finalize()
    prog.launch(prog.io())
    return out


def _pick_kp(k: int, choices, tp: int) -> int:
    for kp in choices:
        if tp * kp <= MAX_PARTS and k % kp == 0 and (k // kp) % 64 == 0:
            return kp
    raise ValueError(f"no K part count fits k={k} at tp={tp}")


def fuse_o_proj(cfg, ncta: int, splits: int) -> bool:
    """o_proj runs fused behind the attention stage (``PRO_ATTN``) when every (kv head,
    split) task has a CTA of its own and the heads are 128-dim (the 4B architecture)."""
    return splits > 0 and cfg.num_kv_heads * splits <= ncta and cfg.head_dim == 128 and not cfg.spark_features


def default_order(cfg, ncta: int, tp: int = 1, splits: int = 0, batch: int = 1) -> dict:
    """Slice / part counts of the decode program (the oracle's persistent-step order).

    ``cfg`` is the rank's local config (heads, intermediate size and vocab divided by
    ``tp``); ``splits`` its attention splits per kv head (0: unknown, no fusion).
    "kp_local" are the K parts of o_proj / down on one rank; "kp" the parts of the whole
    model (tp x kp_local: rank r's parts follow rank r - 1's), which is the order the
    oracle restates.  A fused o_proj (``fuse_o_proj``) is cut into one K part per kv head,
    one slice per unit.  Batch programs (``batch`` > 1) never fuse o_proj."""
    h, i, nq, D, v = cfg.hidden_size, cfg.intermediate_size, cfg.num_q_heads, cfg.head_dim, cfg.vocab_size
    fused = batch == 1 and fuse_o_proj(cfg, ncta, splits)
    kp_o = cfg.num_kv_heads if fused else _pick_kp(nq * D, (2, 1), tp)
    kp_down = _pick_kp(i, (4, 2, 1), tp)
    qkv_n = (nq + 2 * cfg.num_kv_heads) * D
    return {
        # 2 slices per unit elsewhere: measured on the 36-layer step, 2 beats 4 (per-task
        # overhead) and 1 (a warp per unit: 11 units in use at once overflow the ring)
        "ks": (pick_ks(qkv_n, h, 1, 2, ncta), 1 if fused else pick_ks(h, nq * D, kp_o, 2, ncta),
               pick_ks(2 * i, h, 1, 2, ncta), pick_ks(h, i, kp_down, 2, ncta), pick_ks(v, h, 1, 2, ncta)),
        "kp": (tp * kp_o, tp * kp_down),
        "kp_local": (kp_o, kp_down),
        "chunk_accs": CHUNK_ACCS,
        "fused_o": fused,
    }


SHORT_SPLITS = 18  # splits per kv head when the context allows (see splits_for)


def splits_for(nkv: int, ncta: int, max_seq_len: int = 0, head_dim: int = 128) -> int:
    """Splits per kv head.  A context that fits takes SHORT_SPLITS (fewer when the CTAs
    cannot give every (kv head, split) task its own CTA): an attention task is bound by its
    latency chain, not by its K / V bytes, so more, shorter splits only add per-task cost
    (q load, merge, combine over more partials).  Measured at ctx 2048: 8 kv heads x 128
    dims best at 18 (12, 9 worse), 4 x 128 (tensor parallel over 2) the same at 18 and 37,
    4 x 256 best at 18-24 (27, 32, 37 worse).  Longer contexts take the fewest splits that
    hold them, rounded up to whole rounds of tasks over the CTAs (8 kv heads: 37 = 296
    tasks = two per CTA, ...) so no CTA runs a round more than the others."""
    need = max(1, -(-max_seq_len // MAX_SPLIT_TOKENS))
    one_round = max(1, min(ncta // nkv, MAX_SPLITS))
    short = min(one_round, SHORT_SPLITS)
    if need <= short:
        return short
    rounds = max(1, -(-need * nkv // ncta))
    splits = max(need, rounds * ncta // nkv)
    if splits > MAX_SPLITS:
        raise ValueError(f"max_seq_len {max_seq_len} needs {splits} splits per kv head (limit {MAX_SPLITS})")
    return splits


def batch_splits(nkv: int, ncta: int, max_seq_len: int, batch: int) -> int:
    """Splits per kv head of a batch-B program: the fewest that hold the context, rounded
    up to whole rounds of the B x nkv x splits tasks over the CTAs."""
    need = max(1, -(-max_seq_len // MAX_SPLIT_TOKENS))
    pairs = nkv * batch
    rounds = max(1, -(-need * pairs // ncta))
    splits = max(need, rounds * ncta // pairs)
    if splits > MAX_SPLITS:
        raise ValueError(f"max_seq_len {max_seq_len} needs {splits} splits per kv head (limit {MAX_SPLITS})")
    return splits


def attn_splits(cfg, ncta: int, max_seq_len: int = 0) -> int:
    """Splits per kv head of ``cfg`` (the rank's local config under tensor parallelism)."""
    return splits_for(cfg.num_kv_heads, ncta, max_seq_len, cfg.head_dim)


def max_split_tokens(max_seq_len: int, splits: int) -> int:
    return (math.ceil(max_seq_len / splits) + 15) // 16 * 16
