"""Q6_K LM head over a tied embedding (the Spark checkpoint's ``token_embd``).

Mirrors the reference's ``Q6HeadMethod`` / ``install`` (integration/head.py:6-31; the
repack of tools/deployment/prepare_head.py:11-28): the vocab embedding stays vLLM's
(bf16 weight, ``F.embedding``), and the LM-head projection of one decode token
(x bf16 [1, hidden]) runs on the original Q6_K codes -- here the persistent step
kernel's Q6_K GEMV stage over the T6 layout (``spark_q6k_pack_t6``), one cooperative
launch, bf16 logits.  Other shapes (prefill, batches) take vLLM's bf16 path.  The
reference checks that the layer's bf16 weight is the Q6_K decode of the same codes;
``install_q6_head`` does the same check (on the device, against
``spark_q6k_dequantize``) before it swaps the method in.
"""
from __future__ import annotations

import ctypes

import torch
from vllm.model_executor.layers.vocab_parallel_embedding import UnquantizedEmbeddingMethod

from .. import ops
from .. import step as S
from .._lib import SparkStage, call


class SparkQ6HeadMethod(UnquantizedEmbeddingMethod):
    """``apply`` for one bf16 token: the Q6_K GEMV (T6 units in ``layer.spark_q6_t6``)."""

    def __init__(self, vocab: int, hidden: int, ks: int = 4):
        super().__init__()
        self.vocab, self.hidden, self.ks = vocab, hidden, ks

    def _stage(self, w: torch.Tensor, x: torch.Tensor, y: torch.Tensor) -> SparkStage:
        st = SparkStage()
        st.kind, st.pro, st.epi, st.rowmap = S.STAGE_GEMV_Q6, S.PRO_BF16, S.EPI_BF16, S.ROWS_PLAIN
        st.n, st.k, st.kp, st.ks = self.vocab, self.hidden, 1, self.ks
        st.units, st.rot, st.wait = self.vocab // 16, 0, -1
        st.w, st.a, st.out = ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(
            y.data_ptr())
        return st

    def apply(self, layer, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
        t6 = getattr(layer, "spark_q6_t6", None)
        if (t6 is None or bias is not None or x.dim() != 2 or x.shape[0] != 1 or x.shape[1] != self.hidden or
                x.dtype != torch.bfloat16 or not x.is_cuda):
            return super().apply(layer, x, bias)
        xc = x.contiguous()
        y = torch.empty((1, self.vocab), dtype=torch.bfloat16, device=x.device)
        st = self._stage(t6, xc, y)
        counters = layer.spark_q6_counters
        io = S.SparkStepIO()
        io.counters, io.tp_size = ctypes.c_void_p(counters.data_ptr()), 1
        call("spark_step_run", ctypes.byref(st), None, 1, ctypes.byref(io), S._stream())
        return y


def install_q6_head(head: torch.nn.Module, q6k_blocks: torch.Tensor, ks: int = 4) -> SparkQ6HeadMethod:
    """Swap a vocab embedding / LM head (``weight`` bf16 [vocab, hidden] on the GPU) to
    the Q6_K decode method.  ``q6k_blocks``: the same weight's gguf Q6_K rows, uint8
    [vocab, hidden / 256 * 210].  Refuses when the bf16 weight is not the Q6_K decode
    of those codes (the reference's tied-embedding check, integration/head.py:26-27)."""
    w = head.weight
    vocab, hidden = w.shape
    blocks = q6k_blocks.to(w.device).contiguous()
    if vocab % 16 or hidden % 256 or blocks.numel() != vocab * hidden // 256 * 210:
        raise ValueError(f"Q6_K head needs vocab % 16 == 0, hidden % 256 == 0 and matching blocks "
                         f"(got {tuple(w.shape)}, {blocks.numel()} bytes)")
    deq = ops.q6k_dequantize(blocks).view(vocab, hidden)
    if not torch.equal(deq.to(torch.bfloat16).view(torch.int16), w.detach().to(torch.bfloat16).view(torch.int16)):
        raise ValueError("the embedding weight is not the bf16 decode of these Q6_K codes")
    head.register_buffer("spark_q6_t6", S.q6k_pack_t6(blocks, vocab, hidden), persistent=False)
    head.register_buffer("spark_q6_counters", torch.zeros(4, dtype=torch.int32, device=w.device), persistent=False)
    method = SparkQ6HeadMethod(vocab, hidden, ks)
    head.quant_method = method
    return method
