"""vLLM plugin entry point of the B200 decode path (``vllm.general_plugins``).

Mirrors the reference plugin (src/spark_vllm_ascend/plugin/__init__.py:60-87, entry
point pyproject.toml:13-14): ``register()`` is called by vLLM in the API server,
engine-core and worker processes, must be cheap and idempotent, and this module
imports only the standard library so that loading the entry point never pulls in
torch or CUDA.  ``register()`` then wires, lazily:

* the quantization method ``spark_q4_0`` (``SparkQ4Config`` / ``SparkQ4LinearMethod``,
  Q4_0 GEMV on sm_100a through ``torch.ops.spark_b200.q4_gemv``);
* the attention backend ``SparkAttentionBackend`` into vLLM's CUSTOM backend slot
  (paged split-KV decode attention over BF16 K / V, 128-token pages stored one
  (block, kv head) page contiguous).

Set ``SPARK_B200_PLUGIN_DISABLE=1`` to make ``register()`` stand down (the reference's
override switch, inverted: this plugin adds kernels, not a model architecture).
"""
from __future__ import annotations

import logging
import os

logger = logging.getLogger(__name__)

QUANT_NAME = "spark_q4_0"
BACKEND_PATH = "spark_b200.plugin.attention.SparkAttentionBackend"
DISABLE_ENV = "SPARK_B200_PLUGIN_DISABLE"
TESTED_VLLM = "0.22.0"

_registered = False


def _disabled() -> bool:
    return os.environ.get(DISABLE_ENV, "").strip().lower() in ("1", "true", "yes", "on")


def register() -> None:
    """Register the Spark B200 quantization method and attention backend with vLLM."""
    global _registered
    if _registered:
        return
    if _disabled():
        logger.info("spark_b200 plugin: %s set, standing down", DISABLE_ENV)
        return
    import vllm
    from vllm.v1.attention.backends.registry import AttentionBackendEnum, register_backend

    from . import quant  # noqa: F401  (registers spark_q4_0 on import)

    register_backend(AttentionBackendEnum.CUSTOM, BACKEND_PATH)
    _registered = True
    logger.info("spark_b200 plugin: registered quantization %s and attention backend %s "
                "(tested against vLLM %s, running %s)", QUANT_NAME, BACKEND_PATH, TESTED_VLLM, vllm.__version__)


def is_registered() -> bool:
    return _registered
