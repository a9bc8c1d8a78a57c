"""spark_b200 -- B200-native (sm_100a) batch-1 decode hot path of the Spark vLLM plugin.

Subpackages / modules:
  _lib      ctypes binding of libspark_b200.so (C ABI, include/spark_b200.h)
  ops       torch-facing operators and torch.ops.spark_b200.* registrations
  config    SparkConfig (synthetic 4B decoder by default)
  model     synthetic weights, paged KV cache and the CUDA-graph decode engine
  plugin    vLLM general-plugin entry point (registration only)
"""
from __future__ import annotations

__version__ = "0.1.0"


def ensure_built() -> None:
    """Build libspark_b200.so when it is missing (needs nvcc; no GPU required)."""
    from ._lib import library_path

    if not library_path().exists():
        import importlib.util
        from pathlib import Path

        build_py = Path(__file__).resolve().parents[1] / "build.py"
        spec = importlib.util.spec_from_file_location("spark_b200_build", build_py)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()
