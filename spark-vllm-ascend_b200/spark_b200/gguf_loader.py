"""Load a Spark GGUF checkpoint into the decode engine's weights.

Follows the reference's loader (src/spark_vllm_ascend/integration/weights.py:10-82):

* ``verify``: the file's size and sha256 against ``DOWNLOAD_VERIFIED.json`` beside it
  (and an expected sha256, when given), as ``reader()`` does (weights.py:12-20);
* tensor names as in ``hf_name`` (weights.py:22-29): ``token_embd``, ``output_norm``,
  ``blk.{i}.attn_norm`` / ``ffn_norm`` (F32), ``attn_qkv`` (fused q / k / v rows, or
  separate ``attn_q`` / ``attn_k`` / ``attn_v``), ``attn_gate`` (the headwise output
  gate's rows), ``attn_output``, ``ffn_gate`` / ``ffn_up`` / ``ffn_down`` -- Q4_0 blocks,
  split losslessly into the engine's planes on the GPU (``spark_q4_split_gguf``; the
  reference's ``unpack_q4``, weights.py:34-40);
* the tied Q6_K ``token_embd``: its gguf decode (``spark_q6k_dequantize``, bf16) is the
  embedding and its codes are the LM head (the reference's Q6 head, head.py:6-31);
  a float embedding with a Q4_0 ``output`` tensor is the untied alternative.

The reference repacks into its megakernel tiles on the host and keeps that form; here
the T16 / T6 packing runs on the GPU when ``DecodeEngine`` is built (milliseconds for
the 2.4 GB), so nothing repacked is cached on disk.  The GGUF is read with gguf 0.19.0
(the reference's pinned reader).
"""
from __future__ import annotations

import hashlib
import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from . import ops
from .config import SparkConfig
from .model import BF16, LayerWeights, Q4Linear, SyntheticWeights, rope_cos_sin

Q4_0, Q6_K, F32, F16, BF16_T = 2, 14, 0, 1, 30


def verify(path, sha256: str | None = None) -> dict:
    """Size and sha256 of ``path`` against ``DOWNLOAD_VERIFIED.json`` beside it (when
    present) and against ``sha256`` (when given); raises ValueError on a mismatch.  With
    neither, the file is not hashed (``sha256`` None in the result)."""
    p = Path(path)
    size = p.stat().st_size
    rec = p.with_name("DOWNLOAD_VERIFIED.json")
    if sha256 is None and not rec.exists():  # nothing to check against: skip the hash
        return {"size": size, "sha256": None}
    h = hashlib.sha256()
    with open(p, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 24), b""):
            h.update(chunk)
    digest = h.hexdigest()
    if rec.exists():
        v = json.loads(rec.read_text())
        if int(v.get("size", size)) != size:
            raise ValueError(f"{p.name}: size {size} != recorded {v['size']}")
        if v.get("sha256", digest) != digest:
            raise ValueError(f"{p.name}: sha256 {digest} != recorded {v['sha256']}")
    if sha256 is not None and sha256 != digest:
        raise ValueError(f"{p.name}: sha256 {digest} != expected {sha256}")
    return {"size": size, "sha256": digest}


@dataclass
class _T:
    name: str
    kind: int
    rows: int
    cols: int
    data: np.ndarray  # raw bytes [rows, row bytes] (quantized) or values


def _tensors(reader) -> dict[str, _T]:
    out = {}
    for t in reader.tensors:
        shape = [int(v) for v in t.shape]  # gguf order: columns first
        cols = shape[0]
        rows = int(np.prod(shape[1:])) if len(shape) > 1 else 1
        out[t.name] = _T(t.name, int(t.tensor_type), rows, cols, np.asarray(t.data))
    return out


def _need(ts: dict, name: str, kinds: tuple, rows: int | None, cols: int | None) -> _T:
    t = ts.get(name)
    if t is None:
        raise KeyError(f"GGUF tensor {name} missing")
    if t.kind not in kinds:
        raise ValueError(f"{name}: type {t.kind}, expected one of {kinds}")
    if (rows is not None and t.rows != rows) or (cols is not None and t.cols != cols):
        raise ValueError(f"{name}: shape [{t.rows}, {t.cols}], expected [{rows}, {cols}]")
    return t


def plan(reader, cfg: SparkConfig) -> dict:
    """Check every tensor the engine needs against ``cfg`` (names, types, shapes), on
    the host; returns the tensors by role.  Raises KeyError / ValueError."""
    ts = _tensors(reader)
    h, i, nq, nkv, D, V = (cfg.hidden_size, cfg.intermediate_size, cfg.num_q_heads, cfg.num_kv_heads,
                           cfg.head_dim, cfg.vocab_size)
    fl = (F32, F16, BF16_T)
    out = {"layers": []}
    for li in range(cfg.num_layers):
        p = f"blk.{li}."
        lay = {"in_norm": _need(ts, p + "attn_norm.weight", fl, 1, h),
               "post_norm": _need(ts, p + "ffn_norm.weight", fl, 1, h)}
        if p + "attn_qkv.weight" in ts:
            lay["qkv"] = [_need(ts, p + "attn_qkv.weight", (Q4_0,), (nq + 2 * nkv) * D, h)]
        else:
            lay["qkv"] = [_need(ts, p + "attn_q.weight", (Q4_0,), nq * D, h),
                          _need(ts, p + "attn_k.weight", (Q4_0,), nkv * D, h),
                          _need(ts, p + "attn_v.weight", (Q4_0,), nkv * D, h)]
        if cfg.attn_gate:
            lay["gate"] = _need(ts, p + "attn_gate.weight", (Q4_0,), nq, h)
        lay["o"] = _need(ts, p + "attn_output.weight", (Q4_0,), h, nq * D)
        lay["gate_up"] = [_need(ts, p + "ffn_gate.weight", (Q4_0,), i, h), _need(ts, p + "ffn_up.weight", (Q4_0,), i, h)]
        lay["down"] = _need(ts, p + "ffn_down.weight", (Q4_0,), h, i)
        out["layers"].append(lay)
    out["final_norm"] = _need(ts, "output_norm.weight", fl, 1, h)
    if cfg.tied_q6k_head:
        out["embed_q6"] = _need(ts, "token_embd.weight", (Q6_K,), V, h)
    else:
        out["embed"] = _need(ts, "token_embd.weight", fl, V, h)
        out["head"] = _need(ts, "output.weight", (Q4_0,), V, h)
    return out


class GGUFWeights(SyntheticWeights):
    """The engine's weights from a GGUF file (same attributes as ``SyntheticWeights``:
    ``layers`` of Q4_0 planes, ``embed``, ``final_norm``, ``head`` or ``head_q6``,
    RoPE tables), uploaded to ``device`` and split there."""

    def __init__(self, path, cfg: SparkConfig, device="cuda", sha256: str | None = None,
                 expect_tensors: int | None = None, check: bool = True):
        import gguf
        self.cfg = cfg
        self.device = torch.device(device)
        self.path = str(path)
        self.verified = verify(path, sha256) if check else None
        reader = gguf.GGUFReader(str(path))
        if expect_tensors is not None and len(reader.tensors) != expect_tensors:
            raise ValueError(f"{path}: {len(reader.tensors)} tensors, expected {expect_tensors}")
        pl = plan(reader, cfg)
        dev = self.device

        def up(a: np.ndarray) -> torch.Tensor:
            return torch.from_numpy(np.array(a, order="C")).to(dev)  # (a copy: the file map is read-only)

        def q4(parts: list) -> Q4Linear:
            k = parts[0].cols
            rows = sum(t.rows for t in parts)
            blocks = up(np.concatenate([t.data.reshape(t.rows, -1) for t in parts]))
            qs, d = ops.q4_split_gguf(blocks, rows, k)
            return Q4Linear(qs, d)

        def vec(t: _T) -> torch.Tensor:
            return up(t.data.astype(np.float32).reshape(-1)).to(BF16)

        self.layers = []
        for lay in pl["layers"]:
            qkv = q4(lay["qkv"])
            if cfg.attn_gate:  # the gate logits' rows after the heads, zero rows up to 16
                g = q4([lay["gate"]])
                pad = cfg.gate_rows - g.n
                qkv = Q4Linear(torch.cat([qkv.qs, g.qs, torch.zeros((pad, g.qs.shape[1]), dtype=torch.uint8,
                                                                     device=dev)]),
                               torch.cat([qkv.d, g.d, torch.zeros((pad, g.d.shape[1]), dtype=g.d.dtype, device=dev)]))
            self.layers.append(LayerWeights(in_norm=vec(lay["in_norm"]), post_norm=vec(lay["post_norm"]), qkv=qkv,
                                            o=q4([lay["o"]]), gate_up=q4(lay["gate_up"]), down=q4([lay["down"]])))
        self.final_norm = vec(pl["final_norm"])
        if cfg.tied_q6k_head:
            t = pl["embed_q6"]
            self.head_q6 = up(t.data.reshape(t.rows, -1))
            self.embed = ops.q6k_dequantize(self.head_q6).view(cfg.vocab_size, cfg.hidden_size).to(BF16)
            self.head = None
        else:
            self.head_q6 = None
            self.embed = up(pl["embed"].data.astype(np.float32).reshape(cfg.vocab_size, -1)).to(BF16)
            self.head = q4([pl["head"]])
        self.cos_sin = rope_cos_sin(cfg, theta=cfg.rope_theta, rotary_dim=cfg.rotary_dim or None).to(dev)
        self.cos_sin_sliding = None
        if any(cfg.is_sliding(li) for li in range(cfg.num_layers)):
            self.cos_sin_sliding = rope_cos_sin(cfg, theta=cfg.rope_theta_sliding or cfg.rope_theta).to(dev)


def load_gguf(path, cfg: SparkConfig | None = None, device="cuda", **kw) -> GGUFWeights:
    """``GGUFWeights`` of ``path``; ``cfg`` defaults to the Spark-X2.6-4B architecture."""
    if cfg is None:
        from .config import spark_x26_config
        cfg = spark_x26_config()
    return GGUFWeights(path, cfg, device=device, **kw)
