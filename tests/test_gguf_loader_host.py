"""Host-side checks of the GGUF loader (spark_b200.gguf_loader): the download record
check (the reference's reader(), integration/weights.py:12-20) and the tensor plan's
errors for missing tensors and wrong shapes, on small files written with gguf's writer."""
from __future__ import annotations

import json

import numpy as np
import pytest


def _write(path, tensors: dict):
    import gguf
    wr = gguf.GGUFWriter(str(path), "spark2_5")
    for name, (arr, kind) in tensors.items():
        wr.add_tensor(name, arr, raw_dtype=kind)
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()


def _tiny(tmp_path, drop=None, bad=None):
    import gguf
    from spark_b200.config import spark_x26_config
    Q = gguf.GGMLQuantizationType
    cfg = spark_x26_config(num_layers=1, hidden_size=256, num_q_heads=4, num_kv_heads=1, intermediate_size=512,
                           vocab_size=32, layer_types=("full_attention",))
    h, i, D = 256, 512, 256
    q4 = lambda n, k: (np.zeros((n, k // 32 * 18), np.uint8), Q.Q4_0)  # noqa: E731
    f32 = lambda n: (np.ones(n, np.float32), Q.F32)  # noqa: E731
    t = {"blk.0.attn_norm.weight": f32(h), "blk.0.ffn_norm.weight": f32(h),
         "blk.0.attn_qkv.weight": q4(6 * D, h), "blk.0.attn_gate.weight": q4(4, h),
         "blk.0.attn_output.weight": q4(h, 4 * D), "blk.0.ffn_gate.weight": q4(i, h),
         "blk.0.ffn_up.weight": q4(i, h), "blk.0.ffn_down.weight": q4(h, i), "output_norm.weight": f32(h),
         "token_embd.weight": (np.zeros((32, 210), np.uint8), Q.Q6_K)}
    if drop:
        t.pop(drop)
    if bad:
        t[bad] = q4(16, h)
    p = tmp_path / "m.gguf"
    _write(p, t)
    return p, cfg


def test_plan_accepts_spark_layout(tmp_path):
    import gguf
    from spark_b200 import gguf_loader
    p, cfg = _tiny(tmp_path)
    pl = gguf_loader.plan(gguf.GGUFReader(str(p)), cfg)
    assert pl["layers"][0]["qkv"][0].rows == 6 * 256 and pl["embed_q6"].rows == 32


def test_plan_reports_missing_and_misshaped(tmp_path):
    import gguf
    from spark_b200 import gguf_loader
    p, cfg = _tiny(tmp_path, drop="blk.0.ffn_up.weight")
    with pytest.raises(KeyError, match="ffn_up"):
        gguf_loader.plan(gguf.GGUFReader(str(p)), cfg)
    p, cfg = _tiny(tmp_path, bad="blk.0.attn_output.weight")
    with pytest.raises(ValueError, match="attn_output"):
        gguf_loader.plan(gguf.GGUFReader(str(p)), cfg)


def test_verify_download_record(tmp_path):
    import hashlib
    from spark_b200 import gguf_loader
    p, _ = _tiny(tmp_path)
    data = p.read_bytes()
    sha = hashlib.sha256(data).hexdigest()
    assert gguf_loader.verify(p, sha)["size"] == len(data)
    assert gguf_loader.verify(p)["sha256"] is None  # no record, no expected digest: not hashed
    rec = tmp_path / "DOWNLOAD_VERIFIED.json"
    rec.write_text(json.dumps({"size": len(data), "sha256": sha}))
    assert gguf_loader.verify(p)["sha256"] == sha
    rec.write_text(json.dumps({"size": len(data), "sha256": "0" * 64}))
    with pytest.raises(ValueError, match="sha256"):
        gguf_loader.verify(p)
    rec.write_text(json.dumps({"size": len(data) + 1, "sha256": sha}))
    with pytest.raises(ValueError, match="size"):
        gguf_loader.verify(p)
    rec.unlink()
    with pytest.raises(ValueError, match="expected"):
        gguf_loader.verify(p, "1" * 64)
