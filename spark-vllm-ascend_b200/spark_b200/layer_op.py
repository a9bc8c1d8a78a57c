"""The reference's per-layer decode op on the persistent step kernel.

The reference serves batch-1 decode through one torch custom op per decoder layer,
``spark_v43::layer_run(x, residual, positions, key) -> (x, residual)``
(src/spark_vllm_ascend/integration/model.py:46-82), which its model's forward calls in a
loop over the layers (plugin/spark2_5.py:369-376).  ``x`` is the layer's normalized input
(the previous layer's next-norm, or the first input_layernorm), ``residual`` the residual
stream before the layer's attention; the op runs attention and the MLP and returns the
next layer's normalized input and the new residual.  The KV cache is written through a
side channel (``mutates_args=()`` with the cache found by ``key``), as in the reference.

``torch.ops.spark_b200.layer_run`` keeps that contract.  ``key`` names a ``LayerBinding``
registered with ``register_layer`` (the reference finds its layer through vLLM's forward
context, ``get_attention_context(key)``, model.py:49; a caller inside vLLM registers the
binding once per layer with the layer's weights, KV cache and block table).  One call is
ONE persistent launch (``spark_step_run``) of a four-stage program -- qkv GEMV + RoPE +
paged K / V store; split-KV attention with o_proj fused behind it; post-attention
add + RMSNorm + gate_up GEMV + SiLU * mul; down GEMV -- followed by the next norm
(``spark_add_rmsnorm``).  The whole model in one launch per token is
``spark_b200.model.DecodeEngine(mode="step")``; this op is the per-layer boundary the
reference's model class calls.
"""
from __future__ import annotations

import torch

from . import ops
from . import step as S

BF16 = torch.bfloat16


class LayerBinding:
    """Everything ``layer_run`` needs for one decoder layer (persistent device buffers, so
    the program's pointers stay valid and the op can be captured in a CUDA graph).

    ``lw``: the layer's Q4_0 weights (``.qkv``, ``.o``, ``.gate_up``, ``.down`` with
    ``.qs`` / ``.d`` planes) and ``.post_norm``; ``next_norm``: the gamma of the norm the
    op applies last (the next layer's input norm, or the final norm); ``k_cache`` /
    ``v_cache``: this layer's paged caches bf16 [blocks][nkv][block_size][head_dim];
    ``block_table`` int32 (the sequence's logical -> physical blocks, device)."""

    def __init__(self, cfg, lw, next_norm: torch.Tensor, cos_sin: torch.Tensor, k_cache: torch.Tensor,
                 v_cache: torch.Tensor, block_table: torch.Tensor, max_seq_len: int, rotary_dim: int = 0):
        if cfg.spark_features:
            raise ValueError("layer_run covers the SwiGLU / 128-dim architecture; the Spark layer features run "
                             "in the whole-step engine")
        dev = k_cache.device
        self.cfg = cfg
        h, i, nq, nkv, D, bs = (cfg.hidden_size, cfg.intermediate_size, cfg.num_q_heads, cfg.num_kv_heads,
                                cfg.head_dim, cfg.block_size)
        self.ncta = S.num_ctas()
        self.splits = S.attn_splits(cfg, self.ncta, max_seq_len)
        self.max_split_tokens = S.max_split_tokens(max_seq_len, self.splits)
        order = S.default_order(cfg, self.ncta, 1, self.splits)
        self.order = order
        ks_qkv, ks_o, ks_gu, ks_down, _ = order["ks"]
        kp_o = order["kp_local"][0]
        ks_down = S.pick_ks(h, i, 1, 2, self.ncta)  # down as whole rows (bf16 out for the next norm)
        self.order_down = (1, ks_down)
        e = lambda *s, dt=BF16: torch.zeros(s, dtype=dt, device=dev)  # noqa: E731
        self.x_in, self.res_in = e(h), e(h)
        self.pos = e(1, dt=torch.int64)
        self.q, self.kv_new = e(nq, D), e(2, nkv, D)
        self.part_o, self.part_lse = e(self.splits, nq, D, dt=torch.float32), e(self.splits, nq, dt=torch.float32)
        self.head_ctr = e(nkv, dt=torch.int32)
        self.attn_out = e(nq, D)
        self.o_parts = e(kp_o, h, dt=torch.float32)
        self.res1, self.mid, self.down_out = e(h), e(i), e(h)
        self.y, self.res2 = e(h), e(h)
        self.error = e(1, dt=torch.int32)
        self.next_norm, self.post_norm = next_norm, lw.post_norm
        self.block_table, self.k_cache, self.v_cache, self.cos_sin = block_table, k_cache, v_cache, cos_sin
        self.t16 = (S.q4_pack_t16(lw.qkv.qs, lw.qkv.d, 1, S.ROWS_PAIR_HALF, D, rotary_dim),
                    S.q4_pack_t16(lw.o.qs, lw.o.d, kp_o),
                    S.q4_pack_t16(lw.gate_up.qs, lw.gate_up.d, 1, S.ROWS_GATE_UP),
                    S.q4_pack_t16(lw.down.qs, lw.down.d, 1))
        wq, wo, wgu, wd = self.t16
        rope = {"cos_sin": cos_sin, "pos": self.pos, "block_table": block_table, "k_cache": k_cache,
                "v_cache": v_cache, "q": self.q, "kv_new": self.kv_new, "block_size": bs, "nq": nq, "nkv": nkv}
        prog = S.StepProgram(dev, self.ncta)
        qkv = prog.gemv(wq, cfg.qkv_rows, h, ks=ks_qkv, a=self.x_in, epi=S.EPI_ROPE_KV, rowmap=S.ROWS_PAIR_HALF,
                        head_dim=D, rope=rope, rotary_dim=rotary_dim)
        att = prog.attention(q=self.q, k_cache=k_cache, v_cache=v_cache, kv_new=self.kv_new, block_table=block_table,
                             pos=self.pos, splits=self.splits, max_split_tokens=self.max_split_tokens,
                             scale=cfg.attn_scale, part_o=self.part_o, part_lse=self.part_lse,
                             head_counters=self.head_ctr, attn_out=self.attn_out, nq=nq, nkv=nkv, head_dim=D,
                             block_size=bs, wait=qkv)
        if order["fused_o"]:
            o = prog.gemv(wo, h, nq * D, kp=kp_o, ks=ks_o, epi=S.EPI_PARTS, out=self.o_parts, wait=-1,
                          attn_splits=self.splits)
        else:
            o = prog.gemv(wo, h, nq * D, kp=kp_o, ks=ks_o, a=self.attn_out, epi=S.EPI_PARTS, out=self.o_parts,
                          wait=att)
        gu = prog.gemv(wgu, 2 * i, h, ks=ks_gu, a=self.o_parts, a_parts=kp_o, b=self.res_in, gamma=lw.post_norm,
                       eps=cfg.rms_norm_eps, res_out=self.res1, epi=S.EPI_SILU_MUL, rowmap=S.ROWS_GATE_UP,
                       out=self.mid, wait=o)
        prog.gemv(wd, h, i, kp=1, ks=ks_down, a=self.mid, epi=S.EPI_BF16, out=self.down_out, wait=gu)
        prog.finalize()
        self.program = prog
        self._io = prog.io(error=self.error)

    def reset(self) -> None:
        """Zero the launch counters (after an aborted launch, or before reuse)."""
        self.program.reset_counters()
        self.head_ctr.zero_()
        self.error.zero_()

    def run(self, x: torch.Tensor, residual: torch.Tensor, positions: torch.Tensor):
        h = self.cfg.hidden_size
        if x.dtype != BF16 or residual.dtype != BF16 or x.numel() != h or residual.numel() != h:
            raise ValueError(f"layer_run takes bf16 x / residual of {h} elements (batch-1 decode)")
        if positions.numel() != 1:
            raise ValueError("layer_run decodes one token (positions of one element)")
        self.x_in.copy_(x.reshape(-1))
        self.res_in.copy_(residual.reshape(-1))
        self.pos.copy_(positions.reshape(-1).to(torch.int64))
        self.program.launch(self._io)
        ops.add_rmsnorm_out(self.down_out, self.res1, self.next_norm, self.cfg.rms_norm_eps, self.y,
                            res_out=self.res2)
        return self.y.view_as(x).clone(), self.res2.view_as(residual).clone()


_BINDINGS: dict[str, LayerBinding] = {}


def register_layer(key: str, binding: LayerBinding) -> None:
    """Make ``binding`` the layer that ``layer_run(..., key)`` runs."""
    _BINDINGS[key] = binding


def unregister_all() -> None:
    _BINDINGS.clear()


@torch.library.custom_op("spark_b200::layer_run", mutates_args=())
def layer_run(x: torch.Tensor, residual: torch.Tensor, positions: torch.Tensor,
              key: str) -> tuple[torch.Tensor, torch.Tensor]:
    """One decoder layer of batch-1 decode (the reference's ``spark_v43::layer_run``
    contract): (normalized input, residual) -> (next normalized input, residual)."""
    b = _BINDINGS.get(key)
    if b is None:
        raise KeyError(f"layer_run: no layer registered under {key!r}")
    return b.run(x, residual, positions)


@layer_run.register_fake
def _(x, residual, positions, key):
    return torch.empty_like(x), torch.empty_like(residual)
