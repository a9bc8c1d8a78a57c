"""Model configuration of the synthetic Spark decoder.

The field names follow the reference's HF config class ``Spark2_5Config``
(src/spark_vllm_ascend/plugin/spark2_5_config.py:12-69: hidden_size,
num_hidden_layers, num_attention_heads, num_key_value_heads, head_dim,
intermediate_size, vocab_size, rms_norm_eps, rope parameters) so that a config
loaded from a checkpoint maps 1:1.  Defaults are the synthetic 4B model the
build targets: 36 layers, hidden 2560, 32 q / 8 kv heads of 128, SwiGLU 9728,
vocab 151936, RoPE theta 1e6 over the full head, eps 1e-6, paged KV blocks of 128.
"""
from __future__ import annotations

import math
from dataclasses import asdict, dataclass, field

import numpy as np


@dataclass(frozen=True)
class SparkConfig:
    hidden_size: int = 2560
    num_layers: int = 36
    num_q_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 9728
    vocab_size: int = 151936
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1.0e6
    max_position: int = 40960
    block_size: int = 128
    init_std: float = 0.02
    name: str = field(default="spark-synthetic-4b-q4_0")

    def __post_init__(self):
        if self.hidden_size % 32 or self.intermediate_size % 32:
            raise ValueError("hidden and intermediate sizes must be multiples of the Q4_0 block (32)")
        if self.num_q_heads % self.num_kv_heads:
            raise ValueError("query heads must be a multiple of kv heads")
        if self.head_dim % 2:
            raise ValueError("head_dim must be even for neox RoPE")

    @property
    def qkv_rows(self) -> int:
        return (self.num_q_heads + 2 * self.num_kv_heads) * self.head_dim

    @property
    def attn_scale(self) -> float:
        """Softmax scale 1/sqrt(head_dim) rounded to fp32 (what the kernels multiply by)."""
        return float(np.float32(1.0 / math.sqrt(self.head_dim)))

    def layer_q4_bytes(self) -> int:
        h, i = self.hidden_size, self.intermediate_size
        rows_k = [(self.qkv_rows, h), (h, self.num_q_heads * self.head_dim), (2 * i, h), (h, i)]
        return sum(n * k // 32 * 18 for n, k in rows_k)

    def head_q4_bytes(self) -> int:
        return self.vocab_size * self.hidden_size // 32 * 18

    def kv_bytes_per_token(self) -> int:
        """K + V bytes one context token costs per decode step, over all layers."""
        return 2 * self.num_layers * self.num_kv_heads * self.head_dim * 2

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_hf(cls, hf) -> "SparkConfig":
        """Map a HF-style config (Spark2_5Config / LlamaConfig-like object or dict)."""
        get = (lambda k, d=None: hf.get(k, d)) if isinstance(hf, dict) else (lambda k, d=None: getattr(hf, k, d))
        rope = get("rope_parameters") or {}
        theta = get("rope_theta")
        if theta is None and isinstance(rope, dict):
            first = next(iter(rope.values()), {}) if rope and isinstance(next(iter(rope.values())), dict) else rope
            theta = first.get("rope_theta", 1.0e6)
        heads = get("num_attention_heads")
        return cls(hidden_size=get("hidden_size"), num_layers=get("num_hidden_layers"), num_q_heads=heads,
                   num_kv_heads=get("num_key_value_heads", heads),
                   head_dim=get("head_dim") or get("hidden_size") // heads,
                   intermediate_size=get("intermediate_size"), vocab_size=get("vocab_size"),
                   rms_norm_eps=get("rms_norm_eps", 1e-6), rope_theta=float(theta or 1.0e6),
                   max_position=get("max_position_embeddings", 40960))


def tiny_config(**kw) -> SparkConfig:
    """A small config with the same structure, for parity tests."""
    base = dict(hidden_size=256, num_layers=2, num_q_heads=8, num_kv_heads=2, head_dim=128, intermediate_size=512,
                vocab_size=1024, max_position=4096, name="spark-tiny")
    base.update(kw)
    return SparkConfig(**base)
