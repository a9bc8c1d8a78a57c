"""Model configuration of the synthetic Spark decoder.

The field names follow the reference's HF config class ``Spark2_5Config``
(src/spark_vllm_ascend/plugin/spark2_5_config.py:12-69: hidden_size,
num_hidden_layers, num_attention_heads, num_key_value_heads, head_dim,
intermediate_size, vocab_size, rms_norm_eps, rope parameters) so that a config
loaded from a checkpoint maps 1:1.  Defaults are the synthetic 4B model the
build targets: 36 layers, hidden 2560, 32 q / 8 kv heads of 128, SwiGLU 9728,
vocab 151936, RoPE theta 1e6 over the full head, eps 1e-6, paged KV blocks of 128.

The Spark architecture fields (off in the synthetic 4B model) follow the reference's
Spark2_5 layers (plugin/spark2_5.py:60-241, spark2_5_config.py:12-69): the headwise
sigmoid output gate (g_proj, one logit per q head), exact-erf GELU * mul, sliding-window
layers (every layer but each fourth), per-layer-type RoPE (full layers: theta 5e6 over
rotary 64 of the 256 head dims; sliding layers: theta 1e4 over the whole head) and the
tied Q6_K token embedding as LM head.  ``spark_x26_config()`` is the checkpoint the
reference serves (Spark-X2.6-4B: 36 layers, hidden 2560, 16 q / 4 kv heads of 256,
intermediate 10240, vocab 131072).
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
    # Spark architecture features
    attn_gate: bool = False          # headwise sigmoid output gate (gate rows after the qkv heads)
    hidden_act: str = "silu"         # "gelu": exact-erf GELU * mul
    sliding_window: int = 0          # positions a sliding layer attends, current one included
    layer_types: tuple = ()          # per layer "full_attention" / "sliding_attention"; empty: all full
    rotary_dim: int = 0              # full layers' rotated dims per head (0: head_dim)
    rope_theta_sliding: float = 0.0  # sliding layers' RoPE theta (rotary over the whole head)
    tied_q6k_head: bool = False      # the LM head is the Q6_K token embedding

    def __post_init__(self):
        if self.hidden_size % 32 or self.intermediate_size % 32:
            raise ValueError("hidden and intermediate sizes must be multiples of the Q4_0 block (32)")
        if self.num_q_heads % self.num_kv_heads:
            raise ValueError("query heads must be a multiple of kv heads")
        if self.head_dim % 2:
            raise ValueError("head_dim must be even for neox RoPE")
        if self.hidden_act not in ("silu", "gelu"):
            raise ValueError(f"hidden_act {self.hidden_act!r}: silu or gelu")
        if self.layer_types and len(self.layer_types) != self.num_layers:
            raise ValueError("layer_types needs one entry per layer")
        if any(t not in ("full_attention", "sliding_attention") for t in self.layer_types):
            raise ValueError("layer types are full_attention / sliding_attention")

    @property
    def gate_rows(self) -> int:
        """Gate-logit rows after the q / k / v heads (16-row padded), 0 without the gate."""
        return (self.num_q_heads + 15) // 16 * 16 if self.attn_gate else 0

    @property
    def qkv_rows(self) -> int:
        return (self.num_q_heads + 2 * self.num_kv_heads) * self.head_dim + self.gate_rows

    @property
    def spark_features(self) -> bool:
        return (self.attn_gate or self.hidden_act != "silu" or self.sliding_window > 0 or self.tied_q6k_head or
                self.rotary_dim not in (0, self.head_dim) or any(t == "sliding_attention" for t in self.layer_types))

    def is_sliding(self, layer: int) -> bool:
        return bool(self.layer_types) and self.layer_types[layer] == "sliding_attention"

    def layer_rope(self, layer: int) -> tuple[float, int]:
        """(theta, rotary_dim) of a layer."""
        if self.is_sliding(layer):
            return (self.rope_theta_sliding or self.rope_theta), self.head_dim
        return self.rope_theta, (self.rotary_dim or self.head_dim)

    def layer_window(self, layer: int) -> int:
        return self.sliding_window if self.is_sliding(layer) else 0

    @property
    def attn_scale(self) -> float:
        """Softmax scale 1/sqrt(head_dim) rounded to fp32 (what the kernels multiply by)."""
        return float(np.float32(1.0 / math.sqrt(self.head_dim)))

    def layer_q4_bytes(self) -> int:
        h, i = self.hidden_size, self.intermediate_size
        rows_k = [(self.qkv_rows, h), (h, self.num_q_heads * self.head_dim), (2 * i, h), (h, i)]
        return sum(n * k // 32 * 18 for n, k in rows_k)

    def head_q4_bytes(self) -> int:
        """LM-head weight bytes (Q4_0, or the tied Q6_K embedding)."""
        if self.tied_q6k_head:
            return self.vocab_size * self.hidden_size // 256 * 210
        return self.vocab_size * self.hidden_size // 32 * 18

    def kv_bytes_per_token(self) -> int:
        """K + V bytes one context token costs per decode step, over all layers."""
        return 2 * self.num_layers * self.num_kv_heads * self.head_dim * 2

    def kv_bytes_at(self, ctx: int) -> int:
        """K + V bytes one decode step reads at context ``ctx`` (sliding layers read at
        most their window)."""
        per = 2 * self.num_kv_heads * self.head_dim * 2
        return sum(per * (min(ctx, self.layer_window(li)) if self.layer_window(li) else ctx)
                   for li in range(self.num_layers))

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


def spark_x26_config(**kw) -> SparkConfig:
    """The Spark-X2.6-4B architecture (the reference's served checkpoint): every fourth
    layer full attention with partial RoPE (rotary 64, theta 5e6), the others sliding
    (the reference's kernel attends to the last 513 positions, attention.py:124-127;
    RoPE theta 1e4 over all 256 dims), headwise output gate, GELU * mul, tied Q6_K head."""
    layers = kw.pop("num_layers", 36)
    base = dict(hidden_size=2560, num_layers=layers, num_q_heads=16, num_kv_heads=4, head_dim=256,
                intermediate_size=10240, vocab_size=131072, rms_norm_eps=1e-6, rope_theta=5.0e6,
                max_position=40960, name="spark-x2.6-4b-q4_0", attn_gate=True, hidden_act="gelu",
                sliding_window=513, rotary_dim=64, rope_theta_sliding=1.0e4, tied_q6k_head=True,
                layer_types=tuple("sliding_attention" if (li + 1) % 4 else "full_attention" for li in range(layers)))
    base.update(kw)
    return SparkConfig(**base)


def tiny_config(**kw) -> SparkConfig:
    """A small config with the same structure, for parity tests."""
    base = dict(hidden_size=256, num_layers=2, num_q_heads=8, num_kv_heads=2, head_dim=128, intermediate_size=512,
                vocab_size=1024, max_position=4096, name="spark-tiny")
    base.update(kw)
    return SparkConfig(**base)
