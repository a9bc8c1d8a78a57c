"""Tensor parallelism for the persistent decode step (one process per GPU).

The reference serves its model tensor-parallel through vLLM: column-parallel qkv /
gate_up, row-parallel o_proj / down_proj followed by an all-reduce of the hidden
state, KV heads sharded across ranks and a vocab-parallel LM head (the layer
classes its model builds on, src/spark_vllm_ascend/plugin/spark2_5.py:82-160).
Here the same sharding runs inside ONE persistent kernel per rank and step:

* rank r owns q heads [r nq/tp, (r+1) nq/tp), kv heads [r nkv/tp, ...), intermediate
  rows [r i/tp, ...) and vocab rows [r V/tp, ...); qkv, gate_up and the LM head are
  row shards, o_proj and down_proj K shards;
* o_proj and down_proj are *exchange stages*: each rank's epilogue stores its fp32
  parts straight into every rank's exchange window (peer stores over NVLink), after
  which the stage is counted on every rank; the next stage's prologue sums all
  tp x kp parts in rank order.  The LM head's argmax key is maxed into every rank's
  window the same way, so every rank picks the same token;
* there is no separate collective launch: the all-reduce of the reference is the
  exchange inside the step kernel, and its sum is in a fixed order, so a rank's
  results are bit-identical to the single-GPU order with tp x kp parts
  (``step.default_order(..., tp)["kp"]``).

``ExchangeWindow`` holds what peers write (stage counters, the parts buffers, the
key) in device memory from ``spark_window_alloc``; ranks swap CUDA IPC handles over
torch.distributed and map each other's windows (``spark_ipc_open``).
"""
from __future__ import annotations

import ctypes
import dataclasses

import torch

from ._lib import call
from .config import SparkConfig
from .model import LayerWeights, Q4Linear

IPC_HANDLE_BYTES = 64
_ALIGN = 256
_TYPESTR = {torch.int32: "<i4", torch.int64: "<i8", torch.float32: "<f4", torch.uint8: "|u1"}


class _DeviceArray:
    """Raw device memory described by ``__cuda_array_interface__`` (zero-copy view)."""

    def __init__(self, ptr: int, shape: tuple, dtype: torch.dtype):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": _TYPESTR[dtype], "data": (ptr, False),
                                         "version": 3, "strides": None}


def window_layout(fields: list[tuple[str, tuple, torch.dtype]]) -> tuple[dict, int]:
    """Byte offsets (256-byte aligned) of the window's fields and the total size."""
    offsets, off = {}, 0
    for name, shape, dtype in fields:
        n = 1
        for d in shape:
            n *= d
        offsets[name] = off
        off += (n * torch.empty((), dtype=dtype).element_size() + _ALIGN - 1) // _ALIGN * _ALIGN
    return offsets, max(off, _ALIGN)


def gather_handles(handle: bytes, size: int, group=None) -> list[bytes]:
    """Every rank's IPC handle, in rank order (a collective over torch.distributed)."""
    import torch.distributed as dist
    if len(handle) != IPC_HANDLE_BYTES:
        raise ValueError(f"IPC handles are {IPC_HANDLE_BYTES} bytes")
    handles: list = [None] * size
    dist.all_gather_object(handles, bytes(handle), group=group)
    return handles


class ExchangeWindow:
    """One rank's exchange window and its mappings of the peers' windows."""

    def __init__(self, fields: list[tuple[str, tuple, torch.dtype]], device, rank: int, size: int):
        self.device = torch.device(device)
        self.rank, self.size = rank, size
        self.offsets, self.nbytes = window_layout(fields)
        p = ctypes.c_void_p()
        call("spark_window_alloc", self.nbytes, ctypes.byref(p))
        self.ptr = int(p.value)
        self.t = {name: torch.as_tensor(_DeviceArray(self.ptr + self.offsets[name], shape, dtype), device=self.device)
                  for name, shape, dtype in fields}
        self._opened: list[int] = []
        self.peer_table: torch.Tensor | None = None
        self.bases: list[int] = []

    def handle(self) -> bytes:
        buf = (ctypes.c_char * IPC_HANDLE_BYTES)()
        call("spark_ipc_handle", ctypes.c_void_p(self.ptr), buf)
        return bytes(buf)

    def connect(self, handles: list[bytes]) -> None:
        """Map every peer's window (handles[r] = rank r's ``handle()``) and build the
        device table of window bases the kernel reads."""
        if len(handles) != self.size:
            raise ValueError(f"{len(handles)} handles for {self.size} ranks")
        bases = []
        for r, h in enumerate(handles):
            if r == self.rank:
                bases.append(self.ptr)
                continue
            q = ctypes.c_void_p()
            call("spark_ipc_open", ctypes.create_string_buffer(h, IPC_HANDLE_BYTES), ctypes.byref(q))
            self._opened.append(int(q.value))
            bases.append(int(q.value))
        self.bases = bases
        self.peer_table = torch.tensor(bases, dtype=torch.int64).to(self.device)

    def exchange(self, group=None) -> None:
        """All-gather the IPC handles over torch.distributed and connect."""
        self.connect(gather_handles(self.handle(), self.size, group))

    def close(self) -> None:
        """Unmap the peers' windows and free this one (every rank must have stopped
        writing into it: synchronise and barrier first)."""
        for q in self._opened:
            call("spark_ipc_close", ctypes.c_void_p(q))
        self._opened = []
        if self.ptr:
            self.t = {}
            call("spark_window_free", ctypes.c_void_p(self.ptr))
            self.ptr = 0


# ---------------------------------------------------------------------------- sharding
def check_tp(cfg: SparkConfig, tp: int) -> None:
    if tp < 1 or cfg.num_kv_heads % tp or cfg.num_q_heads % tp or cfg.intermediate_size % tp or \
            cfg.vocab_size % tp:
        raise ValueError(f"tp={tp} does not divide the heads / intermediate size / vocab of {cfg.name}")
    if (cfg.vocab_size // tp) % 16 or (cfg.intermediate_size // tp) % 64:
        raise ValueError(f"tp={tp}: vocab shard must be a multiple of 16 rows, intermediate shard of 64")


def local_config(cfg: SparkConfig, tp: int) -> SparkConfig:
    """The per-rank view: heads, intermediate size and vocab divided by tp."""
    check_tp(cfg, tp)
    return dataclasses.replace(cfg, num_q_heads=cfg.num_q_heads // tp, num_kv_heads=cfg.num_kv_heads // tp,
                               intermediate_size=cfg.intermediate_size // tp, vocab_size=cfg.vocab_size // tp,
                               name=f"{cfg.name}-tp{tp}")


def qkv_rows(cfg: SparkConfig, rank: int, tp: int) -> torch.Tensor:
    """Rows of the fused qkv weight rank r owns: its q heads, then k heads, then v heads,
    then (Spark output gate) its q heads' gate rows (the caller pads those to 16)."""
    D, nq, nkv = cfg.head_dim, cfg.num_q_heads, cfg.num_kv_heads
    ql, kl = nq // tp, nkv // tp
    heads = [*range(rank * ql, (rank + 1) * ql), *(nq + h for h in range(rank * kl, (rank + 1) * kl)),
             *(nq + nkv + h for h in range(rank * kl, (rank + 1) * kl))]
    rows = [torch.arange(h * D, (h + 1) * D) for h in heads]
    if cfg.attn_gate:
        g0 = (nq + 2 * nkv) * D
        rows.append(torch.arange(g0 + rank * ql, g0 + (rank + 1) * ql))
    return torch.cat(rows)


def _pad_rows(lin: Q4Linear, rows: int) -> Q4Linear:
    """Zero Q4_0 rows appended up to ``rows`` (the local gate rows' 16-row padding)."""
    n = rows - lin.n
    if n <= 0:
        return lin
    return Q4Linear(torch.cat([lin.qs, torch.zeros((n, lin.qs.shape[1]), dtype=lin.qs.dtype, device=lin.qs.device)]),
                    torch.cat([lin.d, torch.zeros((n, lin.d.shape[1]), dtype=lin.d.dtype, device=lin.d.device)]))


def gate_up_rows(cfg: SparkConfig, rank: int, tp: int) -> torch.Tensor:
    i = cfg.intermediate_size
    il = i // tp
    return torch.cat([torch.arange(rank * il, (rank + 1) * il), torch.arange(i + rank * il, i + (rank + 1) * il)])


def rows_of(lin: Q4Linear, rows: torch.Tensor) -> Q4Linear:
    idx = rows.to(lin.qs.device)
    return Q4Linear(lin.qs.index_select(0, idx).contiguous(), lin.d.index_select(0, idx).contiguous())


def cols_of(lin: Q4Linear, k0: int, k1: int) -> Q4Linear:
    """Columns [k0, k1) (multiples of the 32-element Q4_0 block)."""
    if k0 % 32 or k1 % 32:
        raise ValueError("K shard must align to Q4_0 blocks")
    return Q4Linear(lin.qs[:, k0 // 2:k1 // 2].contiguous(), lin.d[:, k0 // 32:k1 // 32].contiguous())


class ShardWeights:
    """Rank r's weights: the same attributes as ``model.SyntheticWeights`` with the
    local config (embedding, norms and RoPE table replicated)."""

    def __init__(self, full, rank: int, tp: int):
        cfg = full.cfg
        self.full_cfg = cfg
        self.cfg = local_config(cfg, tp)
        self.rank, self.tp = rank, tp
        self.device = full.device
        D, nq, i = cfg.head_dim, cfg.num_q_heads, cfg.intermediate_size
        ko = nq // tp * D
        il = i // tp
        self.vocab_start = rank * (cfg.vocab_size // tp)
        qr, gr = qkv_rows(cfg, rank, tp), gate_up_rows(cfg, rank, tp)
        self.layers = [LayerWeights(in_norm=l.in_norm, post_norm=l.post_norm,
                                    qkv=_pad_rows(rows_of(l.qkv, qr), self.cfg.qkv_rows),
                                    o=cols_of(l.o, rank * ko, (rank + 1) * ko), gate_up=rows_of(l.gate_up, gr),
                                    down=cols_of(l.down, rank * il, (rank + 1) * il)) for l in full.layers]
        self.embed, self.final_norm, self.cos_sin = full.embed, full.final_norm, full.cos_sin
        self.cos_sin_sliding = getattr(full, "cos_sin_sliding", None)
        vl = cfg.vocab_size // tp
        if getattr(full, "head_q6", None) is not None:  # the tied Q6_K head: this rank's vocab rows
            self.head, self.head_q6 = None, full.head_q6[self.vocab_start:self.vocab_start + vl].contiguous()
        else:
            self.head_q6 = None
            self.head = rows_of(full.head, torch.arange(self.vocab_start, self.vocab_start + vl))

    def layer_cos_sin(self, li: int) -> torch.Tensor:
        return self.cos_sin_sliding if self.cfg.is_sliding(li) else self.cos_sin

    def q4_bytes(self) -> int:
        head = self.head.nbytes() if self.head is not None else self.head_q6.numel()
        return sum(l.qkv.nbytes() + l.o.nbytes() + l.gate_up.nbytes() + l.down.nbytes() for l in self.layers) + head


def window_fields(cfg_local: SparkConfig, order: dict, num_stages: int, tp: int, tagged: bool = False) -> list:
    """What the peers write into a rank's window: the stage counters, the argmax key and
    the o_proj / down parts of every rank -- counted exchange: fp32 [tp * kp][h], one
    buffer for all layers; tagged exchange: int64 [layers][tp * kp][h] words (fp32 bits |
    launch tag << 32), one buffer per layer so a word is written once per launch and its
    tag names the launch."""
    h, L = cfg_local.hidden_size, cfg_local.num_layers
    kp_o, kp_down = order["kp_local"]
    fields = [("counters", (num_stages + 3,), torch.int32), ("key", (1,), torch.int64)]
    if tagged:
        return fields + [("o_tag", (L, tp * kp_o, h), torch.int64), ("down_tag", (L, tp * kp_down, h), torch.int64)]
    return fields + [("o_parts", (tp * kp_o, h), torch.float32), ("down_parts", (tp * kp_down, h), torch.float32)]


def program_stages(num_layers: int) -> int:
    """Stages of the decode program: 5 per layer and the LM head."""
    return 5 * num_layers + 1
