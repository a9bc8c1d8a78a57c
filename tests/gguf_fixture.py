"""Writes Spark GGUF files for the loader tests (gguf 0.19.0's writer), with the tensor
names of the reference's checkpoint (integration/weights.py:22-29)."""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np


def _f32(bits_u16: np.ndarray) -> np.ndarray:
    return (bits_u16.astype(np.uint32) << 16).view(np.float32)


def write_spark_gguf(path, cfg, w: dict, oracle, record: bool = True, fused_qkv: bool = True) -> Path:
    """``w``: ``SyntheticWeights.to_numpy()`` (fused qkv rows, then the gate rows when the
    config has the output gate); Q4_0 blocks rebuilt from the planes with the oracle's
    gguf join; norms written as F32 (their bf16 values); ``token_embd`` as raw Q6_K when
    the head is the tied Q6_K embedding, else as F32 with a Q4_0 ``output`` tensor.
    ``fused_qkv`` False writes ``attn_q`` / ``attn_k`` / ``attn_v`` instead of ``attn_qkv``."""
    import gguf
    Q = gguf.GGMLQuantizationType
    path = Path(path)
    wr = gguf.GGUFWriter(str(path), "spark2_5")
    nh = (cfg.num_q_heads + 2 * cfg.num_kv_heads) * cfg.head_dim
    i = cfg.intermediate_size
    for li in range(cfg.num_layers):
        p = f"layers.{li}."
        qkv = oracle.q4_join(w[p + "qkv_qs"], w[p + "qkv_d"])
        wr.add_tensor(f"blk.{li}.attn_norm.weight", _f32(w[p + "in_norm"]))
        if fused_qkv:
            wr.add_tensor(f"blk.{li}.attn_qkv.weight", qkv[:nh], raw_dtype=Q.Q4_0)
        else:
            q_rows, kv_rows = cfg.num_q_heads * cfg.head_dim, cfg.num_kv_heads * cfg.head_dim
            wr.add_tensor(f"blk.{li}.attn_q.weight", qkv[:q_rows], raw_dtype=Q.Q4_0)
            wr.add_tensor(f"blk.{li}.attn_k.weight", qkv[q_rows:q_rows + kv_rows], raw_dtype=Q.Q4_0)
            wr.add_tensor(f"blk.{li}.attn_v.weight", qkv[q_rows + kv_rows:nh], raw_dtype=Q.Q4_0)
        if cfg.attn_gate:
            wr.add_tensor(f"blk.{li}.attn_gate.weight", qkv[nh:nh + cfg.num_q_heads], raw_dtype=Q.Q4_0)
        wr.add_tensor(f"blk.{li}.attn_output.weight", oracle.q4_join(w[p + "o_qs"], w[p + "o_d"]), raw_dtype=Q.Q4_0)
        gu = oracle.q4_join(w[p + "gu_qs"], w[p + "gu_d"])
        wr.add_tensor(f"blk.{li}.ffn_gate.weight", gu[:i], raw_dtype=Q.Q4_0)
        wr.add_tensor(f"blk.{li}.ffn_up.weight", gu[i:], raw_dtype=Q.Q4_0)
        wr.add_tensor(f"blk.{li}.ffn_down.weight", oracle.q4_join(w[p + "down_qs"], w[p + "down_d"]),
                      raw_dtype=Q.Q4_0)
        wr.add_tensor(f"blk.{li}.ffn_norm.weight", _f32(w[p + "post_norm"]))
    wr.add_tensor("output_norm.weight", _f32(w["final_norm"]))
    if "head_q6" in w:
        wr.add_tensor("token_embd.weight", w["head_q6"], raw_dtype=Q.Q6_K)
    else:
        wr.add_tensor("token_embd.weight", _f32(w["embed"]))
        wr.add_tensor("output.weight", oracle.q4_join(w["head_qs"], w["head_d"]), raw_dtype=Q.Q4_0)
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
    if record:
        data = path.read_bytes()
        (path.parent / "DOWNLOAD_VERIFIED.json").write_text(
            json.dumps({"size": len(data), "sha256": hashlib.sha256(data).hexdigest()}))
    return path
