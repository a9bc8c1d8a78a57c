"""Small-batch greedy decode: B sequences (2, 4 or 8) through one persistent launch per step.

BASELINE configs[4] asks for batch sizes {1, 2, 4, 8} of batch-1-style decode; the
reference serves batch 1 only (its megakernel takes one token per layer call,
integration/model.py:46-82).  Here the B sequences share every weight byte of a step:
each Q4_0 block's integer MMAs multiply the B sequences' digit columns at once (the
step kernel's batch instantiations, ``SparkStage.batch``), so the weights stream once
per step whatever B is, while each sequence keeps its own position, block table, K / V
pages and attention tasks.  Every sequence's tokens and logits are bit-identical to
decoding it alone with the same program order (``oracle_order``), which is what the
parity tests check against the CPU oracle.

Layout: one paged K / V cache per layer shared by the sequences (each sequence owns
disjoint blocks through its row of ``block_tables``), per-sequence activations
sequence-major ([B][...]).
"""
from __future__ import annotations

import torch

from . import step as S

BF16 = torch.bfloat16


class _SeqView:
    """One sequence of a BatchDecodeEngine seen as a one-sequence engine (the attributes
    ``spark_b200.prefill.prefill`` reads and writes)."""

    def __init__(self, eng: "BatchDecodeEngine", b: int):
        self._e, self._b = eng, b
        self.cfg, self.w, self.device, self.max_seq_len = eng.cfg, eng.w, eng.device, eng.max_seq_len
        self.block_table = eng.block_tables[b]
        self.k_cache, self.v_cache = eng.k_cache, eng.v_cache
        self.logits = eng.logits[b]
        self.token, self.pos, self.key = eng.token[b:b + 1], eng.pos[b:b + 1], eng.key[b:b + 1]
        self.step_idx = torch.zeros(1, dtype=torch.int32, device=eng.device)
        self.gelu = None

    @property
    def _prefill_w(self):
        return self._e._prefill_w

    @_prefill_w.setter
    def _prefill_w(self, v):
        self._e._prefill_w = v

    def reset(self, pos: int = 0):
        self.pos.fill_(pos)


class BatchDecodeEngine:
    """Greedy decode of ``batch`` sequences of the synthetic 4B architecture together.

    ``weights``: a ``SyntheticWeights`` (Q4_0, head_dim 128, no Spark features); every
    sequence may be ``max_seq_len`` tokens long.  One ``step()`` is one CUDA-graph replay
    of one persistent launch that advances every sequence by one token."""

    def __init__(self, weights, batch: int, max_seq_len: int, splits: int = 0, seed: int = 0,
                 use_graph: bool = True, max_steps: int | None = None, extra_blocks: int = 8):
        cfg = weights.cfg
        if batch not in (2, 4, 8):
            raise ValueError("batch must be 2, 4 or 8 (batch 1 is DecodeEngine)")
        if cfg.spark_features or cfg.head_dim != 128 or getattr(weights, "tp", 1) > 1:
            raise ValueError("batch decode covers the 4B architecture on one GPU")
        self.cfg, self.w, self.batch = cfg, weights, batch
        dev = self.device = weights.device
        self.ncta = S.num_ctas()
        self.max_seq_len = max_seq_len
        self.splits = splits or S.batch_splits(cfg.num_kv_heads, self.ncta, max_seq_len, batch)
        self.max_split_tokens = S.max_split_tokens(max_seq_len, self.splits)
        if self.max_split_tokens > S.MAX_SPLIT_TOKENS:
            raise ValueError(f"{self.splits} splits give {self.max_split_tokens}-token splits "
                             f"(limit {S.MAX_SPLIT_TOKENS})")
        bs, L, nkv, D = cfg.block_size, cfg.num_layers, cfg.num_kv_heads, cfg.head_dim
        self.nblk_seq = (max_seq_len + bs - 1) // bs
        self.num_blocks = batch * self.nblk_seq + extra_blocks
        g = torch.Generator().manual_seed(seed)
        perm = torch.randperm(self.num_blocks, generator=g)[:batch * self.nblk_seq]
        self.block_tables = perm.view(batch, self.nblk_seq).to(torch.int32).to(dev).contiguous()
        self.k_cache = torch.zeros((L, self.num_blocks, nkv, bs, D), dtype=BF16, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        B, h, i, nq = batch, cfg.hidden_size, cfg.intermediate_size, cfg.num_q_heads
        e = lambda *s, dt=BF16: torch.zeros(s, dtype=dt, device=dev)  # noqa: E731
        self.res_attn, self.resmid, self.mid = e(B, h), e(B, h), e(B, i)
        self.q, self.attn_out, self.kv_new = e(B, nq, D), e(B, nq, D), e(B, 2, nkv, D)
        self.part_o = e(B, self.splits, nq, D, dt=torch.float32)
        self.part_lse = e(B, self.splits, nq, dt=torch.float32)
        self.head_ctr = e(L, B, nkv, dt=torch.int32)
        self.logits = e(B, cfg.vocab_size)
        self.key = e(B, dt=torch.int64)
        self.token = e(B, dt=torch.int32)
        self.pos = e(B, dt=torch.int64)
        self.step_idx = e(1, dt=torch.int32)
        self.max_steps = max_steps or max_seq_len
        self.token_log = e(self.max_steps, B, dt=torch.int32)
        self.error = e(1, dt=torch.int32)
        self.use_graph = use_graph
        self.graph = None
        self._prefill_w = None
        self._build_program()

    def _build_program(self):
        cfg, w, dev, B = self.cfg, self.w, self.device, self.batch
        h, i, nq, nkv, D, bs = (cfg.hidden_size, cfg.intermediate_size, cfg.num_q_heads, cfg.num_kv_heads,
                                cfg.head_dim, cfg.block_size)
        order = S.default_order(cfg, self.ncta, 1, self.splits, batch=B)
        self.step_order = order
        ks_qkv, ks_o, ks_gu, ks_down, ks_head = order["ks"]
        kp_o, kp_down = order["kp_local"]
        self.t16 = [(S.q4_pack_t16(lw.qkv.qs, lw.qkv.d, 1, S.ROWS_PAIR_HALF, D),
                     S.q4_pack_t16(lw.o.qs, lw.o.d, kp_o),
                     S.q4_pack_t16(lw.gate_up.qs, lw.gate_up.d, 1, S.ROWS_GATE_UP),
                     S.q4_pack_t16(lw.down.qs, lw.down.d, kp_down)) for lw in w.layers]
        self.t16_head = S.q4_pack_t16(w.head.qs, w.head.d, 1)
        f32 = torch.float32
        self.o_parts = torch.zeros((B, kp_o, h), dtype=f32, device=dev)
        self.down_parts = torch.zeros((B, kp_down, h), dtype=f32, device=dev)
        prog = S.StepProgram(dev, self.ncta, batch=B, bt_stride=self.nblk_seq)
        eps = cfg.rms_norm_eps
        prev = -1
        for li, (lw, (wq, wo, wgu, wd)) in enumerate(zip(w.layers, self.t16)):
            kc, vc = self.k_cache[li], self.v_cache[li]
            rope = {"cos_sin": w.cos_sin, "pos": self.pos, "block_table": self.block_tables, "k_cache": kc,
                    "v_cache": vc, "q": self.q, "kv_new": self.kv_new, "block_size": bs, "nq": nq, "nkv": nkv}
            src = ({"embed": w.embed, "token": self.token} if li == 0 else
                   {"a": self.down_parts, "a_parts": kp_down, "b": self.resmid})
            qkv = prog.gemv(wq, cfg.qkv_rows, h, ks=ks_qkv, gamma=lw.in_norm, eps=eps, res_out=self.res_attn,
                            epi=S.EPI_ROPE_KV, rowmap=S.ROWS_PAIR_HALF, head_dim=D, rope=rope, wait=prev, **src)
            att = prog.attention(q=self.q, k_cache=kc, v_cache=vc, kv_new=self.kv_new, block_table=self.block_tables,
                                 pos=self.pos, splits=self.splits, max_split_tokens=self.max_split_tokens,
                                 scale=cfg.attn_scale, part_o=self.part_o, part_lse=self.part_lse,
                                 head_counters=self.head_ctr[li], attn_out=self.attn_out, nq=nq, nkv=nkv, head_dim=D,
                                 block_size=bs, wait=qkv)
            o = prog.gemv(wo, h, nq * D, kp=kp_o, ks=ks_o, a=self.attn_out, epi=S.EPI_PARTS, out=self.o_parts,
                          wait=att)
            gu = prog.gemv(wgu, 2 * i, h, ks=ks_gu, a=self.o_parts, a_parts=kp_o, b=self.res_attn,
                           gamma=lw.post_norm, eps=eps, res_out=self.resmid, epi=S.EPI_SILU_MUL,
                           rowmap=S.ROWS_GATE_UP, out=self.mid, wait=o)
            prev = prog.gemv(wd, h, i, kp=kp_down, ks=ks_down, a=self.mid, epi=S.EPI_PARTS, out=self.down_parts,
                             wait=gu)
        prog.gemv(self.t16_head, cfg.vocab_size, h, ks=ks_head, a=self.down_parts, a_parts=kp_down, b=self.resmid,
                  gamma=w.final_norm, eps=eps, epi=S.EPI_ARGMAX, out=self.logits, key=self.key, wait=prev)
        prog.finalize()
        self.program = prog
        self._io = prog.io(error=self.error, key=self.key, token_out=self.token, token_log=self.token_log,
                           step=self.step_idx, pos=self.pos)

    # -- running
    def oracle_order(self) -> dict:
        """The one-sequence oracle order every sequence of this engine follows."""
        return self.step_order

    def _enqueue(self):
        self.program.launch(self._io)

    def capture(self):
        """Capture one step into a CUDA graph (state restored afterwards)."""
        saved = [t.clone() for t in (self.pos, self.step_idx, self.token, self.key)]
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self._enqueue()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._enqueue()
        torch.cuda.synchronize()
        for dst, src in zip((self.pos, self.step_idx, self.token, self.key), saved):
            dst.copy_(src)
        self.graph = g
        return g

    def step(self):
        """Enqueue one decode step of every sequence on the current stream."""
        if self.use_graph:
            if self.graph is None:
                self.capture()
            self.graph.replay()
        else:
            self._enqueue()

    def reset_counters(self):
        """Restart the launch generation (with the head counters it pairs with)."""
        self.program.reset_counters()
        self.head_ctr.zero_()
        self.error.zero_()

    def set_positions(self, pos) -> None:
        self.pos.copy_(torch.as_tensor(pos, dtype=torch.int64).reshape(self.batch))

    def prefill(self, prompts, chunk: int = 2048) -> torch.Tensor:
        """Prefill each sequence's prompt (``spark_b200.prefill``: tensor-core GEMMs over the
        Q4_0 weights, causal attention, K / V into the sequence's own blocks).  Returns the first
        generated token of every sequence (int32 [B])."""
        from .prefill import prefill
        if len(prompts) != self.batch:
            raise ValueError(f"{len(prompts)} prompts for batch {self.batch}")
        self.reset_counters()
        for b, p in enumerate(prompts):
            prefill(_SeqView(self, b), torch.as_tensor(p), chunk)
        self.step_idx.zero_()
        self.key.zero_()
        return self.token.clone()

    def prefill_stepwise(self, prompts) -> torch.Tensor:
        """Feed equal-length prompts one batch step per position (the decode path fills
        the caches; bit-exact with the oracle's token-by-token decode)."""
        P = len(prompts[0])
        if any(len(p) != P for p in prompts) or len(prompts) != self.batch:
            raise ValueError("prefill_stepwise takes batch prompts of one length")
        t = torch.as_tensor(prompts, dtype=torch.int32).to(self.device)  # [B, P]
        self.reset_counters()
        self.pos.zero_()
        self.step_idx.zero_()
        self.key.zero_()
        for i in range(P):
            self.token.copy_(t[:, i])
            self.step()
        return self.token.clone()

    def generate(self, prompts, max_new_tokens: int, stepwise: bool = False) -> list[list[int]]:
        """Greedy decode of every sequence; returns the generated ids per sequence."""
        first = self.prefill_stepwise(prompts) if stepwise else self.prefill(prompts)
        self.step_idx.zero_()
        for _ in range(max_new_tokens - 1):
            self.step()
        torch.cuda.synchronize()
        log = self.token_log[:max_new_tokens - 1].cpu()
        return [[int(first[b])] + log[:, b].tolist() for b in range(self.batch)]
