"""CPU checks of the vLLM plugin surface: the entry point, registration of the
quantization method and attention backend with vLLM 0.22, weight creation and
metadata building.  No kernel is launched here (GPU parity: test_gpu_plugin.py)."""
from __future__ import annotations

import subprocess
import sys
import tomllib
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "spark-vllm-ascend_b200"

vllm = pytest.importorskip("vllm")


def test_entry_point_declared():
    meta = tomllib.loads((PKG / "pyproject.toml").read_text())
    eps = meta["project"]["entry-points"]["vllm.general_plugins"]
    assert eps["spark_b200"] == "spark_b200.plugin:register"


def test_plugin_module_imports_stdlib_only():
    code = ("import sys; import spark_b200.plugin as p; "
            "print(','.join(m for m in ('torch', 'vllm', 'numpy') if m in sys.modules))")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, check=True,
                         env={"PYTHONPATH": str(PKG), "PATH": "/usr/bin:/bin"})
    assert out.stdout.strip() == ""


def test_register_is_idempotent_and_registers_quant_and_backend():
    from spark_b200 import plugin
    from vllm.model_executor.layers.quantization import get_quantization_config
    from vllm.v1.attention.backends.registry import AttentionBackendEnum
    plugin.register()
    plugin.register()
    assert plugin.is_registered()
    cfg_cls = get_quantization_config("spark_q4_0")
    assert cfg_cls.get_name() == "spark_q4_0" and cfg_cls.get_min_capability() == 100
    assert AttentionBackendEnum.CUSTOM.get_path() == plugin.BACKEND_PATH
    from spark_b200.plugin.attention import SparkAttentionBackend
    assert AttentionBackendEnum.CUSTOM.get_class() is SparkAttentionBackend


def test_register_stands_down_when_disabled():
    code = ("import os; os.environ['SPARK_B200_PLUGIN_DISABLE']='1'; import spark_b200.plugin as p; "
            "p.register(); print(p.is_registered())")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, check=True,
                         env={"PYTHONPATH": str(PKG), "PATH": "/usr/bin:/bin"})
    assert out.stdout.strip().splitlines()[-1] == "False"


def test_linear_method_creates_gguf_block_weights():
    import torch
    from spark_b200.plugin.quant import SparkQ4Config, SparkQ4LinearMethod
    m = SparkQ4Config.from_config({}).get_quant_method(torch.nn.Module(), "x")
    assert m is None  # only linear layers are quantized
    method = SparkQ4LinearMethod(SparkQ4Config())
    layer = torch.nn.Module()
    method.create_weights(layer, 2560, [4096, 1024, 1024], 2560, 6144, torch.bfloat16, weight_loader=lambda *a: None)
    assert layer.qweight.shape == (6144, 2560 // 32 * 18) and layer.qweight.dtype == torch.uint8
    assert layer.qweight.input_dim == 1 and layer.qweight.output_dim == 0 and callable(layer.qweight.weight_loader)
    with pytest.raises(ValueError):
        method.create_weights(torch.nn.Module(), 100, [64], 100, 64, torch.bfloat16)


def test_attention_backend_layout_and_metadata():
    import torch
    from spark_b200.plugin.attention import (SparkAttentionBackend, SparkAttentionImpl, SparkAttentionMetadataBuilder,
                                             choose_splits, split_tokens)
    from vllm.v1.attention.backend import AttentionCGSupport, CommonAttentionMetadata
    B = SparkAttentionBackend
    assert B.get_kv_cache_shape(10, 128, 8, 128) == (2, 10, 8, 128, 128)
    assert B.get_supported_kernel_block_sizes() == [128] and B.get_supported_head_sizes() == [128, 256]
    assert B.get_impl_cls() is SparkAttentionImpl and B.get_builder_cls() is SparkAttentionMetadataBuilder
    assert B.get_kv_cache_block_dim(128, 8, 128) == 1
    assert SparkAttentionMetadataBuilder._cudagraph_support == AttentionCGSupport.UNIFORM_SINGLE_TOKEN_DECODE
    assert choose_splits(40960) == 256 and choose_splits(512) == 16 and split_tokens(6144, 48) == 128
    builder = SparkAttentionMetadataBuilder.__new__(SparkAttentionMetadataBuilder)
    builder.splits, builder.max_split_tokens = 16, 128
    cm = CommonAttentionMetadata(
        query_start_loc=torch.tensor([0, 1, 2], dtype=torch.int32), query_start_loc_cpu=torch.tensor([0, 1, 2]),
        seq_lens=torch.tensor([300, 17], dtype=torch.int32), num_reqs=2, num_actual_tokens=2, max_query_len=1,
        max_seq_len=300, block_table_tensor=torch.zeros((2, 4), dtype=torch.int32),
        slot_mapping=torch.tensor([299, 16], dtype=torch.int64))
    md = builder.build(0, cm)
    assert md.is_decode and md.num_reqs == 2 and md.splits == 16 and md.slot_mapping.tolist() == [299, 16]
    impl = SparkAttentionImpl(32, 128, 128 ** -0.5, 8)
    assert impl.num_kv_heads == 8
    with pytest.raises(ValueError):
        SparkAttentionImpl(32, 64, 0.125, 8)
    with pytest.raises(NotImplementedError):  # windows: the head_size-256 (Spark) path only
        SparkAttentionImpl(32, 128, 0.1, 8, sliding_window=512)
    assert SparkAttentionImpl(16, 256, 0.0625, 4, sliding_window=512).window == 513
    with pytest.raises(NotImplementedError):  # head_size 256 takes 4 query heads per kv head
        SparkAttentionImpl(16, 256, 0.0625, 8)


def test_layer_run_op_registered_with_fake():
    """torch.ops.spark_b200.layer_run exists with the reference's signature and a fake
    implementation (no GPU, no library call: meta tensors)."""
    import torch
    from spark_b200 import layer_op  # noqa: F401  (registers the op)
    op = torch.ops.spark_b200.layer_run
    x = torch.empty((1, 2560), dtype=torch.bfloat16, device="meta")
    pos = torch.empty((1,), dtype=torch.int64, device="meta")
    y, r = op(x, x, pos, "model.layers.0.self_attn")
    assert y.shape == (1, 2560) and r.shape == (1, 2560) and y.dtype == torch.bfloat16
