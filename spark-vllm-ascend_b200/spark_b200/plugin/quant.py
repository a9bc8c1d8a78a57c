"""Quantization method ``spark_q4_0``: Q4_0 linear layers on the B200 kernels.

Replaces the reference's quantized linear path (the packed Q4_0 layer weights fed to
its DecodeLayer megakernel, integration/weights.py:42-82, and the quant-method
pattern of integration/head.py:6-31).  Checkpoint tensors are gguf Q4_0 blocks
(uint8 [rows, K/32 * 18]: fp16 scale + 16 nibble bytes per 32 weights), exactly what
vLLM's gguf loader yields; they are sharded by whole rows (column parallel) or by
whole 32-element blocks (row parallel), and split once after loading into the two
planes the kernels read (``spark_q4_split_gguf``, lossless).

Decode tokens (up to 8 rows of x) go through the fused Q4_0 GEMV
(``torch.ops.spark_b200.q4_gemv``); longer inputs (prefill) dequantize to bf16 on the
GPU and use a bf16 matmul.
"""
from __future__ import annotations

from typing import Any

import torch
from vllm.model_executor.layers.linear import LinearBase, LinearMethodBase
from vllm.model_executor.layers.quantization import register_quantization_config
from vllm.model_executor.layers.quantization.base_config import QuantizationConfig
from vllm.model_executor.utils import set_weight_attrs

from .. import ops

BLOCK = 32
BLOCK_BYTES = 18
GEMV_MAX_ROWS = 8


@register_quantization_config("spark_q4_0")
class SparkQ4Config(QuantizationConfig):
    """Q4_0 weights (gguf block format) executed by the sm_100a Q4_0 GEMV."""

    def __init__(self) -> None:
        super().__init__()

    def __repr__(self) -> str:
        return "SparkQ4Config()"

    @classmethod
    def get_name(cls) -> str:
        return "spark_q4_0"

    @classmethod
    def get_supported_act_dtypes(cls) -> list[torch.dtype]:
        return [torch.bfloat16]

    @classmethod
    def get_min_capability(cls) -> int:
        return 100  # sm_100a kernels only

    @staticmethod
    def get_config_filenames() -> list[str]:
        return []

    @classmethod
    def from_config(cls, config: dict[str, Any]) -> "SparkQ4Config":
        return cls()

    def get_quant_method(self, layer: torch.nn.Module, prefix: str):
        if isinstance(layer, LinearBase):
            return SparkQ4LinearMethod(self)
        return None


class SparkQ4LinearMethod(LinearMethodBase):
    """create_weights: ``qweight`` uint8 [out, in/32 * 18] (gguf Q4_0 blocks);
    after loading: ``qs`` uint8 [out, in/2] and ``d`` fp16 [out, in/32]."""

    def __init__(self, quant_config: SparkQ4Config):
        self.quant_config = quant_config

    def create_weights(self, layer: torch.nn.Module, input_size_per_partition: int,
                       output_partition_sizes: list[int], input_size: int, output_size: int,
                       params_dtype: torch.dtype, **extra_weight_attrs):
        if input_size_per_partition % BLOCK:
            raise ValueError(f"spark_q4_0: input size per partition {input_size_per_partition} is not a multiple "
                             f"of the Q4_0 block ({BLOCK})")
        out = sum(output_partition_sizes)
        qweight = torch.nn.Parameter(torch.empty(out, input_size_per_partition // BLOCK * BLOCK_BYTES,
                                                 dtype=torch.uint8), requires_grad=False)
        set_weight_attrs(qweight, {"input_dim": 1, "output_dim": 0})
        set_weight_attrs(qweight, extra_weight_attrs)
        layer.register_parameter("qweight", qweight)
        layer.spark_in = input_size_per_partition
        layer.spark_out = out

    def process_weights_after_loading(self, layer: torch.nn.Module) -> None:
        blocks = layer.qweight.data
        qs, d = ops.q4_split_gguf(blocks.contiguous(), layer.spark_out, layer.spark_in)
        layer.register_buffer("qs", qs, persistent=False)
        layer.register_buffer("d", d, persistent=False)
        # the gguf copy is no longer needed on the device
        layer.qweight = torch.nn.Parameter(torch.empty(0, dtype=torch.uint8, device=blocks.device),
                                           requires_grad=False)

    def apply(self, layer: torch.nn.Module, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).to(torch.bfloat16)
        if x2.shape[0] <= GEMV_MAX_ROWS:
            y = torch.ops.spark_b200.q4_gemv(x2.contiguous(), layer.qs, layer.d)
        else:  # prefill: dequantize on the GPU, bf16 matmul
            w = ops.q4_dequantize(layer.qs, layer.d)
            y = x2 @ w.t()
        if bias is not None:
            y = y + bias
        return y.reshape(*shape[:-1], y.shape[-1])
