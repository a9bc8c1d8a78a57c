"""Synthetic Spark decoder on B200: weights in HBM, paged KV cache and the decode engine.

Structure of one decode step (the reference's per-layer megakernel,
kernels/layer.py:48-103, re-cut into stream-ordered sm_100a kernels launched with
programmatic dependent launch and replayed as one CUDA graph):

  per layer i:
    qkv      : s = a + b -> res_attn; x = RMSNorm(s) * in_norm; QKV Q4 GEMV; RoPE;
               q -> q_buf, k / v -> paged cache at the step's slot
               (layer 0: a = embedding row of the input token, b = none)
    attn     : split-KV attention; the last split CTA of each kv head merges the
               partials (log-sum-exp) -> attn_out (bf16)
    o_proj   : Q4 GEMV attn_out -> oproj
    gate_up  : s = oproj + res_attn -> resmid; x = RMSNorm(s) * post_norm;
               gate/up Q4 GEMV; SiLU(g) * u -> mid
    down     : Q4 GEMV mid -> down          (next layer: a = down, b = resmid)
  head       : s = down + resmid; x = RMSNorm(s) * final_norm; LM-head Q4 GEMV;
               bf16 logits + greedy argmax key
  finalize   : token = argmax; token_log[step] = token; pos += 1; step += 1

This is the same dataflow as the reference's layer_run custom op
(integration/model.py:46-82), whose inputs are the normalised hidden state and the
residual and whose outputs are the next layer's normalised input and residual.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import numpy as np
import torch

from . import ops
from ._lib import lib
from .config import SparkConfig

BF16 = torch.bfloat16


# ---------------------------------------------------------------------------- RoPE table
def rope_cos_sin(cfg: SparkConfig, max_position: int | None = None, theta: float | None = None,
                 rotary_dim: int | None = None) -> torch.Tensor:
    """bf16 [max_pos, r]: cos(pos * inv_freq) | sin(pos * inv_freq), neox layout over the
    r rotated dims (r = head_dim, or a Spark layer type's rotary_dim, with its theta).

    Same construction as vLLM's RotaryEmbedding._compute_cos_sin_cache (fp32 on the
    CPU, then cast to the model dtype), which the reference feeds to its kernel as
    ``cs`` (integration/model.py:71)."""
    max_pos = max_position or cfg.max_position
    d = rotary_dim or cfg.head_dim
    th = theta or cfg.rope_theta
    inv_freq = 1.0 / (th ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
    t = torch.arange(max_pos, dtype=torch.float32)
    freqs = torch.einsum("i,j->ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1).to(BF16).contiguous()


# ---------------------------------------------------------------------------- weights
@dataclass
class Q4Linear:
    qs: torch.Tensor  # uint8 [n, k/2]
    d: torch.Tensor   # fp16 [n, k/32]

    @property
    def n(self) -> int:
        return self.qs.shape[0]

    @property
    def k(self) -> int:
        return self.qs.shape[1] * 2

    def nbytes(self) -> int:
        return self.qs.numel() + self.d.numel() * 2


@dataclass
class LayerWeights:
    in_norm: torch.Tensor
    post_norm: torch.Tensor
    qkv: Q4Linear
    o: Q4Linear
    gate_up: Q4Linear
    down: Q4Linear


class SyntheticWeights:
    """Seeded random-init weights of the synthetic model, generated on the GPU.

    Linear weights are N(0, init_std) in fp32, quantized to Q4_0 on the device by
    ``spark_q4_quantize`` (bit-identical to gguf's quantizer).  Embeddings are bf16
    N(0, init_std).  RMSNorm weights are bf16(1 + N(0, init_std)).

    Spark architecture (``cfg.spark_features``): the qkv rows end with the gate rows;
    with ``tied_q6k_head`` the token embedding is random gguf Q6_K rows (``head_q6``,
    d ~ N(0, init_std / 32)) whose decode is the bf16 embedding and whose codes are the
    LM head; ``cos_sin`` serves the full layers and ``cos_sin_sliding`` the sliding ones.
    """

    def __init__(self, cfg: SparkConfig, device="cuda", seed: int = 0):
        self.cfg = cfg
        self.device = torch.device(device)
        gen = torch.Generator(device=self.device)
        gen.manual_seed(seed)
        std = cfg.init_std
        h, i = cfg.hidden_size, cfg.intermediate_size

        def q4(n, k):
            qs = torch.empty((n, k // 2), dtype=torch.uint8, device=self.device)
            d = torch.empty((n, k // 32), dtype=torch.float16, device=self.device)
            rows_per_chunk = max(1, (1 << 27) // k)  # <= 512 MB of fp32 at a time
            for r0 in range(0, n, rows_per_chunk):
                r1 = min(n, r0 + rows_per_chunk)
                w = torch.randn((r1 - r0, k), generator=gen, device=self.device, dtype=torch.float32) * std
                q, s = ops.q4_quantize(w)
                qs[r0:r1].copy_(q)
                d[r0:r1].copy_(s)
            return Q4Linear(qs, d)

        def norm(n):
            return (1.0 + std * torch.randn((n,), generator=gen, device=self.device)).to(BF16)

        self.head_q6 = None
        if cfg.tied_q6k_head:
            if h % 256 or cfg.vocab_size % 16:
                raise ValueError("a Q6_K head needs hidden % 256 == 0 and vocab % 16 == 0")
            nb = cfg.vocab_size * (h // 256)
            blocks = torch.randint(0, 256, (nb, 210), generator=gen, device=self.device, dtype=torch.int32)
            blocks = blocks.to(torch.uint8)
            d = (torch.randn(nb, generator=gen, device=self.device) * (std / 32)).to(torch.float16)
            blocks[:, 208:210] = d.view(torch.uint8).view(nb, 2)
            self.head_q6 = blocks.view(cfg.vocab_size, -1).contiguous()
            self.embed = ops.q6k_dequantize(self.head_q6).view(cfg.vocab_size, h).to(BF16)
        else:
            self.embed = (torch.randn((cfg.vocab_size, h), generator=gen, device=self.device) * std).to(BF16)
        self.layers: list[LayerWeights] = []
        pad0 = cfg.qkv_rows - cfg.gate_rows + cfg.num_q_heads  # gate rows past the q heads: zero
        for _ in range(cfg.num_layers):
            qkv = q4(cfg.qkv_rows, h)
            if cfg.attn_gate:
                qkv.qs[pad0:].zero_()
                qkv.d[pad0:].zero_()
            self.layers.append(LayerWeights(
                in_norm=norm(h), post_norm=norm(h),
                qkv=qkv, o=q4(h, cfg.num_q_heads * cfg.head_dim),
                gate_up=q4(2 * i, h), down=q4(h, i)))
        self.final_norm = norm(h)
        self.head = None if cfg.tied_q6k_head else q4(cfg.vocab_size, h)
        self.cos_sin = rope_cos_sin(cfg, theta=cfg.rope_theta, rotary_dim=cfg.rotary_dim or None).to(self.device)
        self.cos_sin_sliding = None
        if any(cfg.is_sliding(li) for li in range(cfg.num_layers)):
            self.cos_sin_sliding = rope_cos_sin(cfg, theta=cfg.rope_theta_sliding or cfg.rope_theta).to(self.device)

    def layer_cos_sin(self, li: int) -> torch.Tensor:
        return self.cos_sin_sliding if self.cfg.is_sliding(li) else self.cos_sin

    def q4_bytes(self) -> int:
        """Weight bytes a decode step streams (Q4_0 layers + the LM head)."""
        head = self.head.nbytes() if self.head is not None else self.head_q6.numel()
        return sum(l.qkv.nbytes() + l.o.nbytes() + l.gate_up.nbytes() + l.down.nbytes() for l in self.layers) + head

    def to_numpy(self) -> dict:
        """Host copies (uint16 bit patterns for bf16 / fp16) for the CPU checker."""
        def u16(t):
            return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)

        def u8(t):
            return t.detach().contiguous().cpu().numpy()

        out = {"embed": u16(self.embed), "final_norm": u16(self.final_norm), "cos_sin": u16(self.cos_sin)}
        if self.head is not None:
            out["head_qs"], out["head_d"] = u8(self.head.qs), u16(self.head.d)
        if self.head_q6 is not None:
            out["head_q6"] = u8(self.head_q6)
        if self.cos_sin_sliding is not None:
            out["cos_sin_sliding"] = u16(self.cos_sin_sliding)
        for li, l in enumerate(self.layers):
            p = f"layers.{li}."
            out[p + "in_norm"] = u16(l.in_norm)
            out[p + "post_norm"] = u16(l.post_norm)
            for key, lin in (("qkv", l.qkv), ("o", l.o), ("gu", l.gate_up), ("down", l.down)):
                out[p + key + "_qs"] = u8(lin.qs)
                out[p + key + "_d"] = u16(lin.d)
        return out


# ---------------------------------------------------------------------------- engine
def _vp(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def chain_splits(max_seq_len: int) -> int:
    """Attention splits of the kernel chain for contexts up to ``max_seq_len``: 16 while a
    split fits the wide attention kernel (at most 400 tokens: one CTA per split and kv
    head, the split's K / V in shared memory), measured best over ctx 2048 -> 6143 (16 / 24
    / 49 splits: 650 / 596 / 546 tok/s); beyond, splits of at most 128 tokens (one K/V
    chunk), 16 to 256 of them."""
    if -(-max_seq_len // 16) <= 400:
        return 16
    return min(256, max(16, -(-max_seq_len // 128)))


class DecodeEngine:
    """Batch-1 greedy decode of the synthetic model with a paged BF16 KV cache.

    All state lives in HBM; one decode step is one CUDA-graph replay with no host
    synchronisation.  ``block_table`` maps logical KV blocks to physical blocks of
    the cache (a random permutation by default, as in the attention parity cases).
    """

    def __init__(self, weights: SyntheticWeights, max_seq_len: int, splits: int = 0, num_blocks: int | None = None,
                 block_table: torch.Tensor | None = None, use_graph: bool = True, max_steps: int | None = None,
                 seed: int = 0, mode: str = "step", tp_group=None, tp_exchange: str = "counted"):
        """``mode`` "step": one persistent kernel per decode step (spark_b200.step);
        "kernels": the per-stage kernel chain (5 kernels per layer + head + finalize).

        Tensor parallel: ``weights`` is a ``tp.ShardWeights`` (rank r of tp) and every rank
        constructs its engine at the same time (the exchange windows are connected over
        torch.distributed, ``tp_group`` or the default group); persistent step only.
        ``tp_exchange``: "counted" (parts stored to every rank, then a system-scope fence
        and a count on every rank's stage counter; the default, measured faster) or
        "tagged" (parts as 64-bit words carrying the launch number, read once the tags
        match, no fence or counter)."""
        if tp_exchange not in ("counted", "tagged"):
            raise ValueError(f"unknown tp_exchange {tp_exchange!r}")
        self.tp_exchange = tp_exchange
        cfg = weights.cfg
        self.cfg, self.w = cfg, weights
        dev = weights.device
        self.device = dev
        if mode not in ("step", "kernels"):
            raise ValueError(f"unknown mode {mode!r}")
        self.mode = mode
        self.tp_size = getattr(weights, "tp", 1)
        self.tp_rank = getattr(weights, "rank", 0)
        self.tp_group = tp_group
        self.window = None
        if self.tp_size > 1 and mode != "step":
            raise ValueError("tensor parallelism runs on the persistent step (mode='step')")
        if cfg.spark_features and mode != "step":
            raise ValueError("the Spark layer features run on the persistent step (mode='step')")
        if mode == "step":
            from . import step as _step
            self.ncta = _step.num_ctas()
            splits = splits or _step.attn_splits(cfg, self.ncta, max_seq_len)
        if splits <= 0:
            splits = chain_splits(max_seq_len)
        self.splits = splits
        self.max_seq_len = max_seq_len
        bs = cfg.block_size
        nblk_seq = (max_seq_len + bs - 1) // bs
        self.num_blocks = num_blocks or nblk_seq
        if self.num_blocks < nblk_seq:
            raise ValueError("num_blocks too small for max_seq_len")
        self.max_split_tokens = ((max_seq_len + splits - 1) // splits + 15) // 16 * 16
        if self.max_split_tokens > 2048:
            raise ValueError(f"{splits} splits give {self.max_split_tokens}-token splits; use more splits (limit 2048)")
        if block_table is None:
            g = torch.Generator().manual_seed(seed)
            block_table = torch.randperm(self.num_blocks, generator=g)[:nblk_seq].to(torch.int32)
        self.block_table = block_table.to(dev, torch.int32).contiguous()
        L, nkv, D = cfg.num_layers, cfg.num_kv_heads, cfg.head_dim
        self.k_cache = torch.zeros((L, self.num_blocks, nkv, bs, D), dtype=BF16, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        h, i, nq = cfg.hidden_size, cfg.intermediate_size, cfg.num_q_heads
        e = lambda *s, dt=BF16: torch.zeros(s, dtype=dt, device=dev)  # noqa: E731
        self.res_attn, self.resmid, self.oproj, self.down = e(h), e(h), e(h), e(h)
        self.mid = e(i)
        self.q = e(nq, D)
        self.attn_out = e(nq, D)
        self.part_o = e(splits, nq, D, dt=torch.float32)
        self.part_lse = e(splits, nq, dt=torch.float32)
        self.counters = e(cfg.num_kv_heads, dt=torch.int32)
        self.logits = e(cfg.vocab_size)
        self.key = e(1, dt=torch.int64)
        self.token = e(1, dt=torch.int32)
        self.pos = e(1, dt=torch.int64)
        self.step_idx = e(1, dt=torch.int32)
        self.max_steps = max_steps or max_seq_len
        self.token_log = e(self.max_steps, dt=torch.int32)
        self.error = e(1, dt=torch.int32)
        self.use_graph = use_graph
        self.graph = None
        if mode == "step":
            self._build_program()
        else:
            self._calls = self._build_calls()

    # -- the persistent-kernel program of one step
    def _build_program(self):
        from . import step as S
        cfg, w, dev = self.cfg, self.w, self.device
        h, i, nq, nkv, D, bs = (cfg.hidden_size, cfg.intermediate_size, cfg.num_q_heads, cfg.num_kv_heads,
                                cfg.head_dim, cfg.block_size)
        if self.max_split_tokens > S.MAX_SPLIT_TOKENS:
            raise ValueError(f"{self.splits} splits give {self.max_split_tokens}-token splits (limit "
                             f"{S.MAX_SPLIT_TOKENS}); max_seq_len too large for the persistent step")
        tp = self.tp_size
        order = S.default_order(cfg, self.ncta, tp, self.splits)
        fused = order["fused_o"]
        self.step_order = order
        ks_qkv, ks_o, ks_gu, ks_down, ks_head = order["ks"]
        kp_o, kp_down = order["kp_local"]
        # T16 copies of the weights (the gguf planes stay for the per-kernel path)
        self.t16 = []
        rots = [cfg.layer_rope(li)[1] % D for li in range(cfg.num_layers)]  # 0: the whole head
        for lw, rot in zip(w.layers, rots):
            self.t16.append((S.q4_pack_t16(lw.qkv.qs, lw.qkv.d, 1, S.ROWS_PAIR_HALF, D, rot),
                             S.q4_pack_t16(lw.o.qs, lw.o.d, kp_o),
                             S.q4_pack_t16(lw.gate_up.qs, lw.gate_up.d, 1, S.ROWS_GATE_UP),
                             S.q4_pack_t16(lw.down.qs, lw.down.d, kp_down)))
        q6_head = getattr(w, "head_q6", None) is not None
        if q6_head:  # the tied Q6_K embedding as LM head
            self.t16_head = S.q6k_pack_t6(w.head_q6, cfg.vocab_size, h)
        else:
            self.t16_head = S.q4_pack_t16(w.head.qs, w.head.d, 1)
        self.gate = torch.zeros(nq, dtype=BF16, device=dev) if cfg.attn_gate else None
        self.gelu = S.gelu_table(dev) if cfg.hidden_act == "gelu" else None
        f32 = torch.float32
        if tp > 1:  # what peers write lives in the exchange window
            from . import tp as T
            tagged_x = self.tp_exchange == "tagged"
            self.window = T.ExchangeWindow(T.window_fields(cfg, order, T.program_stages(cfg.num_layers), tp,
                                                           tagged_x), dev, self.tp_rank, tp)
            self.window.exchange(self.tp_group)
            self.key = self.window.t["key"]
            if not tagged_x:
                self.o_parts, self.down_parts = self.window.t["o_parts"], self.window.t["down_parts"]
        else:
            self.o_parts = torch.zeros((kp_o, h), dtype=f32, device=dev)
            self.down_parts = torch.zeros((kp_down, h), dtype=f32, device=dev)
        # tensor parallel: o_proj / down parts go to every rank's window, counted (fence +
        # remote counts) or as tagged words (per-layer buffers; readers wait on the tags);
        # the LM head's argmax key is always a counted exchange
        tagged = tp > 1 and self.tp_exchange == "tagged"
        xchg = S.XCHG_TAGGED if tagged else (S.XCHG_COUNTED if tp > 1 else S.XCHG_LOCAL)
        o_out = (lambda li: self.window.t["o_tag"][li]) if tagged else (lambda li: self.o_parts)
        down_out = (lambda li: self.window.t["down_tag"][li]) if tagged else (lambda li: self.down_parts)
        pa_o, pa_down = tp * kp_o, tp * kp_down  # parts the next prologue sums, rank by rank
        self.kv_new = torch.zeros((2, nkv, D), dtype=BF16, device=dev)
        self.head_ctr = torch.zeros((cfg.num_layers, nkv), dtype=torch.int32, device=dev)
        prog = S.StepProgram(dev, self.ncta)
        eps = cfg.rms_norm_eps
        prev = -1
        for li, (lw, (wq, wo, wgu, wd)) in enumerate(zip(w.layers, self.t16)):
            kc, vc = self.k_cache[li], self.v_cache[li]
            cs = w.layer_cos_sin(li) if hasattr(w, "layer_cos_sin") else w.cos_sin
            rope = {"cos_sin": cs, "pos": self.pos, "block_table": self.block_table, "k_cache": kc,
                    "v_cache": vc, "q": self.q, "kv_new": self.kv_new, "block_size": bs, "nq": nq, "nkv": nkv}
            if li == 0:
                src = {"embed": w.embed, "token": self.token}
            else:
                src = {"a": down_out(li - 1), "a_parts": pa_down, "b": self.resmid, "tagged": tagged}
            qkv = prog.gemv(wq, cfg.qkv_rows, h, ks=ks_qkv, gamma=lw.in_norm, eps=eps, res_out=self.res_attn,
                            epi=S.EPI_ROPE_KV, rowmap=S.ROWS_PAIR_HALF, head_dim=D, rope=rope, wait=prev,
                            rotary_dim=rots[li], gate=self.gate, **src)
            att = prog.attention(q=self.q, k_cache=kc, v_cache=vc, kv_new=self.kv_new, block_table=self.block_table,
                                 pos=self.pos, splits=self.splits, max_split_tokens=self.max_split_tokens,
                                 scale=cfg.attn_scale, part_o=self.part_o, part_lse=self.part_lse,
                                 head_counters=self.head_ctr[li], attn_out=self.attn_out, nq=nq, nkv=nkv, head_dim=D,
                                 block_size=bs, wait=qkv, window=cfg.layer_window(li), gate=self.gate)
            if fused:  # o_proj behind the attention, K part = kv head, input in shared memory
                o = prog.gemv(wo, h, nq * D, kp=kp_o, ks=ks_o, epi=S.EPI_PARTS, out=o_out(li), wait=-1,
                              xchg=xchg, attn_splits=self.splits)
            else:
                o = prog.gemv(wo, h, nq * D, kp=kp_o, ks=ks_o, a=self.attn_out, epi=S.EPI_PARTS, out=o_out(li),
                              wait=att, xchg=xchg)
            # gate_up: with tagged parts its wait only orders the residual (written by qkv)
            gu = prog.gemv(wgu, 2 * i, h, ks=ks_gu, a=o_out(li), a_parts=pa_o, b=self.res_attn,
                           gamma=lw.post_norm, eps=eps, res_out=self.resmid,
                           epi=S.EPI_GELU_MUL if self.gelu is not None else S.EPI_SILU_MUL,
                           rowmap=S.ROWS_GATE_UP, out=self.mid, wait=(qkv if tagged else o), table=self.gelu,
                           tagged=tagged)
            down = prog.gemv(wd, h, i, kp=kp_down, ks=ks_down, a=self.mid, epi=S.EPI_PARTS, out=down_out(li),
                             wait=gu, xchg=xchg)
            prev = gu if tagged else down  # what the next reader of the down parts waits on
        prog.gemv(self.t16_head, cfg.vocab_size, h, ks=ks_head, a=down_out(cfg.num_layers - 1), a_parts=pa_down,
                  b=self.resmid, gamma=w.final_norm, eps=eps, epi=S.EPI_ARGMAX, out=self.logits, key=self.key,
                  wait=prev, xchg=S.XCHG_COUNTED if tp > 1 else S.XCHG_LOCAL, row0=getattr(w, "vocab_start", 0),
                  q6=q6_head, tagged=tagged)
        prog.finalize(self.window.t["counters"] if self.window is not None else None)
        self.program = prog
        self._io = prog.io(error=self.error, key=self.key, token_out=self.token, token_log=self.token_log,
                           step=self.step_idx, pos=self.pos, window=self.window)

    # -- the kernel sequence of one step, as prepared ctypes calls (no allocation)
    def _build_calls(self):
        cfg, w = self.cfg, self.w
        L = lib()
        eps = ctypes.c_float(cfg.rms_norm_eps)
        h, i, nq, nkv, D, bs = (cfg.hidden_size, cfg.intermediate_size, cfg.num_q_heads, cfg.num_kv_heads,
                                cfg.head_dim, cfg.block_size)
        scale = ctypes.c_float(cfg.attn_scale)
        layer_stride = self.k_cache[0].numel() * 2
        kc0, vc0 = self.k_cache.data_ptr(), self.v_cache.data_ptr()
        calls = []
        for li, lw in enumerate(w.layers):
            kc = ctypes.c_void_p(kc0 + li * layer_stride)
            vc = ctypes.c_void_p(vc0 + li * layer_stride)
            if li == 0:
                a, b, embed, tok = None, None, _vp(w.embed), _vp(self.token)
            else:
                a, b, embed, tok = _vp(self.down), _vp(self.resmid), None, None
            calls.append((L.spark_qkv_rope_kvstore, "qkv", (
                a, b, embed, tok, _vp(lw.in_norm), eps, _vp(self.res_attn), _vp(lw.qkv.qs), _vp(lw.qkv.d), h, nq,
                nkv, D, _vp(w.cos_sin), _vp(self.pos), _vp(self.block_table), None, bs, kc, vc, _vp(self.q))))
            calls.append((L.spark_attn_decode, "attn", (
                _vp(self.q), kc, vc, _vp(self.block_table), _vp(self.pos), None, nq, nkv, D, bs, self.splits,
                self.max_split_tokens, scale, _vp(self.part_o), _vp(self.part_lse), _vp(self.counters),
                _vp(self.attn_out), _vp(self.error))))
            calls.append((L.spark_q4_gemv, "o_proj", (
                _vp(self.attn_out), _vp(lw.o.qs), _vp(lw.o.d), _vp(self.oproj), h, nq * D, 1)))
            calls.append((L.spark_rmsnorm_gate_up_silu, "gate_up", (
                _vp(self.oproj), _vp(self.res_attn), _vp(lw.post_norm), eps, _vp(self.resmid), _vp(lw.gate_up.qs),
                _vp(lw.gate_up.d), _vp(self.mid), 2 * i, h)))
            calls.append((L.spark_q4_gemv, "down", (
                _vp(self.mid), _vp(lw.down.qs), _vp(lw.down.d), _vp(self.down), h, i, 1)))
        calls.append((L.spark_rmsnorm_q4_head_argmax, "head", (
            _vp(self.down), _vp(self.resmid), _vp(w.final_norm), eps, _vp(w.head.qs), _vp(w.head.d),
            _vp(self.logits), cfg.vocab_size, h, _vp(self.key))))
        calls.append((L.spark_decode_finalize, "finalize", (
            _vp(self.key), _vp(self.token), _vp(self.token_log), _vp(self.step_idx), _vp(self.pos))))
        return calls

    def kernels_per_step(self) -> int:
        return 1 if self.mode == "step" else len(self._calls)

    def _enqueue(self):
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        if self.mode == "step":
            self.program.launch(self._io, stream)
            return
        for fn, name, args in self._calls:
            st = fn(*args, stream)
            if st != 0:
                raise RuntimeError(f"{name}: spark status {st}")

    def capture(self):
        """Capture one decode step into a CUDA graph (state is restored afterwards)."""
        saved = [t.clone() for t in (self.pos, self.step_idx, self.token, self.key)]
        kv_saved = None
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self._enqueue()  # warm-up outside capture (also sets smem attributes)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._enqueue()
        torch.cuda.synchronize()
        for dst, src in zip((self.pos, self.step_idx, self.token, self.key), saved):
            dst.copy_(src)
        del kv_saved
        self.graph = g
        return g

    def _tp_barrier(self):
        import torch.distributed as dist
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.tp_group)

    def reset(self, pos: int = 0):
        """Rewind to position ``pos`` (tensor parallel: collective, every rank calls it)."""
        if self.tp_size > 1:  # no rank may still be writing into a window being zeroed
            self._tp_barrier()
        self.pos.fill_(pos)
        self.step_idx.zero_()
        self.key.zero_()
        self.error.zero_()
        if self.mode == "step":  # launch generation and head counters restart together
            self.program.reset_counters()
            self.head_ctr.zero_()
            if self.window is not None and "o_tag" in self.window.t:  # tags restart with the launch count
                self.window.t["o_tag"].zero_()
                self.window.t["down_tag"].zero_()
        if self.tp_size > 1:
            self._tp_barrier()

    def close(self):
        """Release the exchange window (tensor parallel: collective)."""
        if self.window is not None:
            self.graph = None
            self._tp_barrier()
            self.window.close()
            self._tp_barrier()
            self.window = None

    def oracle_order(self) -> dict | None:
        """The oracle evaluation order this engine's kernels follow (None: per-kernel order)."""
        return self.step_order if self.mode == "step" else None

    def step(self):
        """Enqueue one decode step on the current stream (graph replay when captured)."""
        if self.use_graph:
            if self.graph is None:
                self.capture()
            self.graph.replay()
        else:
            self._enqueue()

    def set_token(self, token: int | torch.Tensor):
        if isinstance(token, torch.Tensor):
            self.token.copy_(token.reshape(1), non_blocking=True)
        else:
            self.token.fill_(int(token))

    def prefill(self, prompt: torch.Tensor | list[int], start_pos: int = 0):
        """Feed prompt tokens one decode step each (KV cache fill through the decode path)."""
        prompt = torch.as_tensor(prompt, dtype=torch.int32).to(self.device)
        self.reset(start_pos)
        for t in range(prompt.numel()):
            self.token.copy_(prompt[t:t + 1])
            self.step()
        # the last step's argmax is the first generated token
        return self.token.clone()

    def prefill_batched(self, prompt: torch.Tensor | list[int], chunk: int = 2048, gemm: str = "q4") -> torch.Tensor:
        """Prefill all prompt tokens of a chunk at once (``spark_b200.prefill``: tensor-core
        GEMMs over the Q4_0 weights, or cuBLAS over cached bf16 ones with gemm="bf16", and
        causal attention: the reference's standard prefill path) instead of one decode
        step per token; single GPU.  Returns the first generated token."""
        if self.tp_size > 1:
            raise ValueError("batched prefill runs on one GPU")
        from .prefill import prefill
        return prefill(self, prompt, chunk, gemm)

    def generate(self, prompt, max_new_tokens: int) -> list[int]:
        """Greedy decode: returns the generated token ids (host list)."""
        first = self.prefill(prompt)
        out = [first]
        self.step_idx.zero_()
        for _ in range(max_new_tokens - 1):
            self.step()
        torch.cuda.synchronize()
        toks = self.token_log[:max_new_tokens - 1].cpu().tolist()
        return [int(first.item())] + toks
