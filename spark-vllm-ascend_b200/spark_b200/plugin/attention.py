"""vLLM attention backend over the B200 split-KV decode kernels.

The reference runs attention inside its DecodeLayer megakernel and reads vLLM's paged
metadata through ``get_attention_context`` (integration/model.py:49, 64-69): the block
table, the slot mapping and the sequence lengths.  This backend supplies the same
metadata to the sm_100a kernels:

* KV cache: ``[2, num_blocks, num_kv_heads, block_size, head_size]`` bf16, i.e. for K
  and for V one (block, kv head) page of 128 tokens x 128 dims contiguous, the layout
  ``spark_attn_splitkv`` streams;
* decode (one query token per request): ``spark_kv_store`` writes this step's k / v at
  the slot mapping, then split-KV attention with the fused log-sum-exp combine per
  request (``spark_attn_decode``); uniform single-token decode batches are CUDA-graph
  capturable;
* head_size 256 and sliding-window layers (the reference's Spark model,
  plugin/spark2_5.py:140-241): decode runs the persistent step kernel's attention stage
  as a one-stage program (``spark_step_run``, its Spark instantiation: 16 lanes per
  token, the window's positions only).  A sliding window of W attends to W + 1
  positions, the current one included, as the reference's kernel does (it masks below
  len - 513 for its 512-window layers, kernels/attention.py:124-127);
* prefill (query length > 1) is not on the decode hot path: causal attention in torch
  over the request's gathered pages, on the GPU.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import ClassVar

import ctypes

import torch
from vllm.v1.attention.backend import (AttentionBackend, AttentionCGSupport, AttentionImpl, AttentionMetadataBuilder,
                                       AttentionType, CommonAttentionMetadata)

from .. import ops

BLOCK_SIZE = 128
HEAD_SIZE = 128
HEAD_SIZES = (128, 256)  # 256: the persistent kernel's attention stage (the Spark model)


def choose_splits(max_model_len: int) -> int:
    """Splits of at most 128 tokens (one cache page), between 16 and 256 (the fused
    combine's limit)."""
    return min(256, max(16, -(-max_model_len // BLOCK_SIZE)))


def split_tokens(max_model_len: int, splits: int) -> int:
    return (math.ceil(max_model_len / splits) + 15) // 16 * 16


@dataclass
class SparkAttentionMetadata:
    num_actual_tokens: int
    num_reqs: int
    max_query_len: int
    max_seq_len: int
    query_start_loc: torch.Tensor  # int32 [num_reqs + 1]
    query_start_loc_cpu: torch.Tensor
    seq_lens: torch.Tensor  # int32 [num_reqs] (device)
    block_table: torch.Tensor  # int32 [num_reqs, max_blocks]
    slot_mapping: torch.Tensor  # int64 [num_tokens]
    splits: int
    max_split_tokens: int

    @property
    def is_decode(self) -> bool:
        return self.max_query_len == 1


class SparkAttentionMetadataBuilder(AttentionMetadataBuilder[SparkAttentionMetadata]):
    _cudagraph_support: ClassVar[AttentionCGSupport] = AttentionCGSupport.UNIFORM_SINGLE_TOKEN_DECODE

    def __init__(self, kv_cache_spec, layer_names, vllm_config, device):
        super().__init__(kv_cache_spec, layer_names, vllm_config, device)
        max_len = vllm_config.model_config.max_model_len if vllm_config is not None else 4096
        self.splits = choose_splits(max_len)
        self.max_split_tokens = split_tokens(max_len, self.splits)

    def build(self, common_prefix_len: int, common_attn_metadata: CommonAttentionMetadata,
              fast_build: bool = False) -> SparkAttentionMetadata:
        cm = common_attn_metadata
        return SparkAttentionMetadata(
            num_actual_tokens=cm.num_actual_tokens, num_reqs=cm.num_reqs, max_query_len=cm.max_query_len,
            max_seq_len=cm.max_seq_len, query_start_loc=cm.query_start_loc, query_start_loc_cpu=cm.query_start_loc_cpu,
            seq_lens=cm.seq_lens, block_table=cm.block_table_tensor, slot_mapping=cm.slot_mapping,
            splits=self.splits, max_split_tokens=self.max_split_tokens)


class SparkAttentionImpl(AttentionImpl[SparkAttentionMetadata]):
    def __init__(self, num_heads: int, head_size: int, scale: float, num_kv_heads: int | None = None,
                 alibi_slopes: list[float] | None = None, sliding_window: int | None = None,
                 kv_cache_dtype: str = "auto", logits_soft_cap: float | None = None,
                 attn_type: str = AttentionType.DECODER, kv_sharing_target_layer_name: str | None = None) -> None:
        if head_size not in HEAD_SIZES:
            raise ValueError(f"SparkAttentionBackend supports head_size {HEAD_SIZES}, got {head_size}")
        if alibi_slopes is not None or logits_soft_cap:
            raise NotImplementedError("SparkAttentionBackend: alibi / soft cap are not supported")
        if sliding_window is not None and head_size != 256:
            raise NotImplementedError("SparkAttentionBackend: sliding windows with head_size 256 only")
        if head_size == 256 and num_heads != 4 * (num_kv_heads or num_heads):
            raise NotImplementedError("SparkAttentionBackend: head_size 256 needs 4 query heads per kv head")
        if attn_type != AttentionType.DECODER:
            raise NotImplementedError("SparkAttentionBackend: decoder self-attention only")
        if kv_cache_dtype not in ("auto", "bfloat16"):
            raise NotImplementedError("SparkAttentionBackend: bf16 KV cache only")
        self.num_heads = num_heads
        self.head_size = head_size
        self.num_kv_heads = num_kv_heads or num_heads
        self.scale = float(scale)
        self.kv_cache_dtype = kv_cache_dtype
        self.kv_sharing_target_layer_name = kv_sharing_target_layer_name
        # positions attended by a sliding layer (the reference's 512-window layers: 513)
        self.window = sliding_window + 1 if sliding_window is not None else 0
        self._ws: dict = {}
        self._step = None

    def _workspace(self, splits: int, device) -> tuple:
        key = (splits, device)
        ws = self._ws.get(key)
        if ws is None:
            nq, d = self.num_heads, self.head_size
            ws = (torch.empty((splits, nq, d), dtype=torch.float32, device=device),
                  torch.empty((splits, nq), dtype=torch.float32, device=device),
                  torch.zeros(self.num_kv_heads, dtype=torch.int32, device=device),  # left zero by the kernel
                  torch.zeros(1, dtype=torch.int32, device=device))
            self._ws[key] = ws
        return ws

    def forward(self, layer, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, kv_cache: torch.Tensor,
                attn_metadata: SparkAttentionMetadata, output: torch.Tensor, output_scale: torch.Tensor | None = None,
                output_block_scale: torch.Tensor | None = None) -> torch.Tensor:
        if attn_metadata is None:  # profiling run
            return output.fill_(0)
        md = attn_metadata
        nq, nkv, d = self.num_heads, self.num_kv_heads, self.head_size
        t = md.num_actual_tokens
        q = query[:t].view(t, nq, d)
        k_cache, v_cache = kv_cache[0], kv_cache[1]
        if self.kv_sharing_target_layer_name is None and key is not None:
            ops.kv_store_(key[:t].view(t, nkv, d), value[:t].view(t, nkv, d), md.slot_mapping[:t], k_cache, v_cache)
        out = output[:t].view(t, nq, d)
        if md.is_decode and (d != HEAD_SIZE or self.window):
            return self._decode_step(q, key, value, k_cache, v_cache, md, out, output)
        if md.is_decode:
            part_o, part_lse, counters, err = self._workspace(md.splits, query.device)
            for r in range(md.num_reqs):  # one query token per request
                ops.attn_decode_out(q[r], k_cache, v_cache, md.block_table[r], md.splits, md.max_split_tokens,
                                    self.scale, part_o, part_lse, counters, out[r], seq_len=md.seq_lens[r:r + 1],
                                    error=err)
            return output
        return self._prefill(q, k_cache, v_cache, md, out, output)

    def _step_state(self, md, device):
        """Persistent buffers of the one-stage step-kernel program (fixed pointers, so a
        captured decode graph replays them): partials, head counters, launch counters,
        this step's k / v per request, positions, the error word."""
        from .. import step as S
        if self._step is None:
            nq, nkv, d = self.num_heads, self.num_kv_heads, self.head_size
            ncta = S.num_ctas()
            max_len = md.splits * md.max_split_tokens  # the builder's bound on the model length
            splits = S.splits_for(nkv, ncta, max_len, d)
            z = lambda *sh, dt=torch.float32: torch.zeros(sh, dtype=dt, device=device)  # noqa: E731
            self._step = {"splits": splits, "T": S.max_split_tokens(max_len, splits), "part_o": z(splits, nq, d),
                          "part_lse": z(splits, nq), "head_ctr": z(nkv, dt=torch.int32),
                          "counters": z(4, dt=torch.int32), "error": z(1, dt=torch.int32), "kv_new": {}, "pos": {}}
        return self._step

    def _decode_step(self, q, key, value, k_cache, v_cache, md, out, output):
        from .. import step as S
        from .._lib import SparkStage, call
        st_ = self._step_state(md, q.device)
        nq, nkv, d, R = self.num_heads, self.num_kv_heads, self.head_size, md.num_reqs
        kvn = st_["kv_new"].get(R)
        if kvn is None:
            kvn = st_["kv_new"][R] = torch.zeros((R, 2, nkv, d), dtype=torch.bfloat16, device=q.device)
            st_["pos"][R] = torch.zeros(R, dtype=torch.int64, device=q.device)
        pos = st_["pos"][R]
        kvn[:, 0].copy_(key[:R].view(R, nkv, d))
        kvn[:, 1].copy_(value[:R].view(R, nkv, d))
        pos.copy_(md.seq_lens[:R])
        pos.sub_(1)
        io = S.SparkStepIO()
        io.counters, io.error, io.tp_size = ctypes.c_void_p(st_["counters"].data_ptr()), \
            ctypes.c_void_p(st_["error"].data_ptr()), 1
        for r in range(R):  # one query token per request
            stg = SparkStage()
            stg.kind, stg.wait = S.STAGE_ATTN, -1
            stg.nq, stg.nkv, stg.head_dim, stg.block_size = nq, nkv, d, k_cache.shape[2]
            stg.splits, stg.max_split_tokens, stg.scale, stg.window = st_["splits"], st_["T"], self.scale, self.window
            for name, tns in (("q", q[r]), ("k_cache", k_cache), ("v_cache", v_cache), ("kv_new", kvn[r]),
                              ("block_table", md.block_table[r]), ("pos", pos[r:r + 1]),
                              ("part_o", st_["part_o"]), ("part_lse", st_["part_lse"]),
                              ("head_counters", st_["head_ctr"]), ("attn_out", out[r])):
                setattr(stg, name, ctypes.c_void_p(tns.data_ptr()))
            call("spark_step_run", ctypes.byref(stg), None, 1, ctypes.byref(io), S._stream())
        return output

    def _prefill(self, q, k_cache, v_cache, md, out, output):
        qsl = md.query_start_loc_cpu.tolist()
        seq = md.seq_lens.tolist()
        group = self.num_heads // self.num_kv_heads
        bs = k_cache.shape[2]
        for r in range(md.num_reqs):
            q0, q1, n = qsl[r], qsl[r + 1], seq[r]
            if q1 <= q0:
                continue
            nblk = -(-n // bs)
            pages = md.block_table[r, :nblk].long()
            kr = k_cache[pages].permute(1, 0, 2, 3).reshape(self.num_kv_heads, nblk * bs, -1)[:, :n]
            vr = v_cache[pages].permute(1, 0, 2, 3).reshape(self.num_kv_heads, nblk * bs, -1)[:, :n]
            kr = kr.repeat_interleave(group, dim=0)
            vr = vr.repeat_interleave(group, dim=0)
            qr = q[q0:q1].transpose(0, 1)  # [nq, lq, d]
            lq = q1 - q0
            # query i sits at absolute position n - lq + i and sees keys 0 .. n - lq + i
            qpos = (n - lq + torch.arange(lq, device=q.device))[:, None]
            kpos = torch.arange(n, device=q.device)[None, :]
            mask = kpos <= qpos
            if self.window:  # (sliding layers: the last `window` positions)
                mask &= kpos > qpos - self.window
            o = torch.nn.functional.scaled_dot_product_attention(qr.float(), kr.float(), vr.float(), attn_mask=mask,
                                                                 scale=self.scale)
            out[q0:q1] = o.transpose(0, 1).to(out.dtype)
        return output


class SparkAttentionBackend(AttentionBackend):
    supported_dtypes: ClassVar[list[torch.dtype]] = [torch.bfloat16]
    supported_kv_cache_dtypes: ClassVar[list] = ["auto", "bfloat16"]
    forward_includes_kv_cache_update: bool = True

    @staticmethod
    def get_name() -> str:
        return "CUSTOM"

    @staticmethod
    def get_impl_cls():
        return SparkAttentionImpl

    @staticmethod
    def get_builder_cls():
        return SparkAttentionMetadataBuilder

    @staticmethod
    def get_kv_cache_shape(num_blocks: int, block_size: int, num_kv_heads: int, head_size: int,
                           cache_dtype_str: str = "auto") -> tuple[int, ...]:
        return (2, num_blocks, num_kv_heads, block_size, head_size)

    @staticmethod
    def get_supported_kernel_block_sizes() -> list[int]:
        return [BLOCK_SIZE]

    @classmethod
    def get_supported_head_sizes(cls) -> list[int]:
        return list(HEAD_SIZES)
