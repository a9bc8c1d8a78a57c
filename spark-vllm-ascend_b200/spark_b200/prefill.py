"""Batched prompt prefill for ``DecodeEngine``: all prompt tokens of a chunk at once.

The reference keeps vLLM's standard PyTorch path for prefill and runs its megakernel
for decode only (integration/model.py:50-62: query length > 1 falls back to the torch
layer); its linear layers multiply by the bf16 dequantization of each Q4_0 weight
(``dequantize(...).bfloat16()``, weights.py:28-31).  This is the same split on B200.  The
four projections of a layer run on the tensor cores straight from the Q4_0 planes
(``gemm="q4"``, the default: ``spark_q4_gemm_tc``, weights dequantized to bf16 in shared
memory, tcgen05 MMAs with fp32 accumulation; no bf16 copy of the weights in HBM), or, with
``gemm="bf16"``, as cuBLAS bf16 GEMMs over a bf16 dequantization made once per engine (2
bytes per weight of HBM, 4.5 GB for the 4B models; kept for later prompts).  Attention is
causal scaled-dot-product attention over the paged cache (the chunk's own K / V are
written into it first), and the element-wise steps follow the decode engine's semantics
(bf16 residual, fp32 RMSNorm, bf16-rounded inputs to the fp32 RoPE, SiLU / GELU of the
bf16 gate, the Spark output gate and sliding window); add + RMSNorm, RoPE and the
activation * mul run as row-batched kernels (``spark_add_rmsnorm_rows``,
``spark_rope_neox_rows``, ``spark_act_mul_rows``, the last with the decode epilogues'
SiLU / GELU-table arithmetic).  Results agree with token-by-token decode within bf16
rounding, not bit for bit (the GEMM summation order is the tensor cores').  After
``prefill`` the engine holds the prompt's K / V, ``pos`` = prompt length and ``token`` =
the first generated token.
"""
from __future__ import annotations

import warnings

import torch
import torch.nn.functional as F

from . import ops

BF16 = torch.bfloat16


def _sdpa(q, K, V, scale, causal, mask=None):
    """q [nq, n, D], K / V [nkv, m, D] bf16 (nq a multiple of nkv) -> [nq, n, D]: a fused
    backend (flash, cuDNN, memory-efficient) with grouped-query heads when one takes the
    shapes, else the kv heads repeated for the fused backends, else the math path."""
    from torch.nn.attention import SDPBackend, sdpa_kernel
    fused = [SDPBackend.FLASH_ATTENTION, SDPBackend.CUDNN_ATTENTION, SDPBackend.EFFICIENT_ATTENTION]
    kw = dict(is_causal=causal, scale=scale) if mask is None else dict(attn_mask=mask, scale=scale)
    rep = q.shape[0] // K.shape[0]
    if rep > 1:
        try:
            with sdpa_kernel(fused), warnings.catch_warnings():
                warnings.simplefilter("ignore")  # (a backend that declines the shapes says why)
                return F.scaled_dot_product_attention(q.unsqueeze(0), K.unsqueeze(0), V.unsqueeze(0),
                                                      enable_gqa=True, **kw)[0]
        except RuntimeError:
            K, V = K.repeat_interleave(rep, 0), V.repeat_interleave(rep, 0)
    args = (q.unsqueeze(0).contiguous(), K.unsqueeze(0).contiguous(), V.unsqueeze(0).contiguous())
    try:
        with sdpa_kernel(fused):
            return F.scaled_dot_product_attention(*args, **kw)[0]
    except RuntimeError:
        return F.scaled_dot_product_attention(*args, **kw)[0]


def _bf16_weights(eng) -> list:
    """Per layer the bf16 dequantization of qkv / o / gate_up / down (made once per
    engine: 2 bytes per weight of HBM, 4.5 GB for the 4B models)."""
    if getattr(eng, "_prefill_w", None) is None:
        deq = ops.q4_dequantize
        eng._prefill_w = [(deq(l.qkv.qs, l.qkv.d), deq(l.o.qs, l.o.d), deq(l.gate_up.qs, l.gate_up.d),
                           deq(l.down.qs, l.down.d)) for l in eng.w.layers]
    return eng._prefill_w


class _Q4Linear:
    """x @ W^T for a Q4_0 weight on the tensor cores (``spark_q4_gemm_tc``); every call
    reports into one device status word that ``check`` reads once per prefill."""

    def __init__(self, device):
        self.err = torch.zeros(1, dtype=torch.int32, device=device)

    def __call__(self, x, q):
        return ops.q4_gemm(x, q.qs, q.d, self.err)

    def check(self):
        e = int(self.err.item())
        if e:
            raise RuntimeError(f"spark_q4_gemm_tc: a wait inside the kernel ran out (status {e})")


def _gather(cache: torch.Tensor, table: torch.Tensor, n: int, bs: int) -> torch.Tensor:
    """Positions [0, n) of one layer's paged cache [blocks, nkv, bs, D] -> [nkv, n, D]."""
    pos = torch.arange(n, device=cache.device)
    return cache[table[pos // bs].long(), :, pos % bs].transpose(0, 1)


@torch.no_grad()
def prefill(eng, prompt: torch.Tensor, chunk: int = 2048, gemm: str = "q4") -> torch.Tensor:
    """Fill ``eng``'s KV cache with ``prompt`` (int32 [P]) from position 0 and set the
    first generated token; returns it (int32 [1]).  ``gemm``: "q4" (tensor-core GEMMs
    over the Q4_0 planes) or "bf16" (cuBLAS over a cached bf16 dequantization)."""
    cfg, w = eng.cfg, eng.w
    dev = eng.device
    prompt = torch.as_tensor(prompt, dtype=torch.int64).to(dev)
    P = prompt.numel()
    if P == 0 or P > eng.max_seq_len:
        raise ValueError(f"prompt of {P} tokens (max_seq_len {eng.max_seq_len})")
    h, i, nq, nkv, D, bs = (cfg.hidden_size, cfg.intermediate_size, cfg.num_q_heads, cfg.num_kv_heads,
                            cfg.head_dim, cfg.block_size)
    nh, eps, scale = nq + 2 * nkv, cfg.rms_norm_eps, cfg.attn_scale
    table = eng.block_table
    if gemm not in ("q4", "bf16"):
        raise ValueError(f"gemm must be 'q4' or 'bf16', not {gemm!r}")
    if gemm == "q4":
        q4 = _Q4Linear(dev)
        mats = [((lambda x, m=l.qkv: q4(x, m)), (lambda x, m=l.o: q4(x, m)), (lambda x, m=l.gate_up: q4(x, m)),
                 (lambda x, m=l.down: q4(x, m))) for l in w.layers]
    else:
        mats = [tuple((lambda x, wt=wt: x @ wt.t()) for wt in ws) for ws in _bf16_weights(eng)]
    heads = torch.arange(nkv, device=dev)
    eng.reset(0)
    a_last = b_last = None
    for p0 in range(0, P, chunk):
        p1 = min(P, p0 + chunk)
        n = p1 - p0
        pos = torch.arange(p0, p1, device=dev)
        a = w.embed[prompt[p0:p1]]  # bf16 [n, h]
        b = None
        for li, (lw, (w_qkv, w_o, w_gu, w_down)) in enumerate(zip(w.layers, mats)):
            res, x = ops.add_rmsnorm_rows(a, b, lw.in_norm, eps)  # (norm of the fp32 sum a + b)
            y = w_qkv(x)
            _, rot = cfg.layer_rope(li)
            cs = w.layer_cos_sin(li) if hasattr(w, "layer_cos_sin") else w.cos_sin
            ops.rope_rows_(y, nq + nkv, D, rot, cs, p0)  # q and k heads, in place
            q = y[:, :nq * D].reshape(n, nq, D)
            k = y[:, nq * D:(nq + nkv) * D].reshape(n, nkv, D)
            v = y[:, (nq + nkv) * D:nh * D].reshape(n, nkv, D)
            # cache rows ((block * nkv + head) * bs + offset) of the chunk's positions
            rows = ((table[pos // bs].long()[:, None] * nkv + heads[None, :]) * bs + (pos % bs)[:, None]).reshape(-1)
            eng.k_cache[li].view(-1, D).index_copy_(0, rows, k.reshape(-1, D))
            eng.v_cache[li].view(-1, D).index_copy_(0, rows, v.reshape(-1, D))
            win = cfg.layer_window(li)
            if p0 == 0:  # the first chunk attends to itself only
                K, V = k.transpose(0, 1), v.transpose(0, 1)  # [nkv, n, D]
            else:
                K = _gather(eng.k_cache[li], table, p1, bs)  # [nkv, p1, D]
                V = _gather(eng.v_cache[li], table, p1, bs)
            if p0 == 0 and (win == 0 or win >= n):  # plain causal: no mask
                o = _sdpa(q.transpose(0, 1), K, V, scale, True)
            else:
                kp = torch.arange(p1, device=dev)
                mask = kp[None, :] <= pos[:, None]
                if win:
                    mask &= kp[None, :] > pos[:, None] - win
                o = _sdpa(q.transpose(0, 1), K, V, scale, False, mask)
            o = o.transpose(0, 1).to(BF16)  # [n, nq, D]
            if cfg.attn_gate:
                g = torch.sigmoid(y[:, nh * D:nh * D + nq].float()).to(BF16)
                o = (o.float() * g.float()[:, :, None]).to(BF16)
            oproj = w_o(o.reshape(n, nq * D))
            resmid, x2 = ops.add_rmsnorm_rows(oproj, res, lw.post_norm, eps)
            gu = w_gu(x2)
            mid = ops.act_mul_rows(gu, getattr(eng, "gelu", None) if cfg.hidden_act == "gelu" else None)
            a = w_down(mid)
            b = resmid
        a_last, b_last = a[-1:], b[-1:]
    # LM head of the last position, greedy
    _, x = ops.add_rmsnorm_rows(a_last, b_last, w.final_norm, eps)
    logits = torch.empty(cfg.vocab_size, dtype=BF16, device=dev)
    if getattr(w, "head_q6", None) is not None:  # Q6_K head: bf16 row chunks and matmul
        rows = 16384
        for r0 in range(0, cfg.vocab_size, rows):
            r1 = min(cfg.vocab_size, r0 + rows)
            wt = ops.q6k_dequantize(w.head_q6[r0:r1].contiguous()).view(r1 - r0, h).to(BF16)
            logits[r0:r1] = (x @ wt.t())[0]
    else:  # one position: the decode path's Q4_0 GEMV, not a dequantized copy of the head
        ops.q4_gemv_out(x, w.head.qs, w.head.d, logits)
    eng.logits.copy_(logits)
    tok = torch.argmax(logits.float()).to(torch.int32).reshape(1)
    if gemm == "q4":
        q4.check()
    eng.token.copy_(tok)
    eng.pos.fill_(P)
    eng.step_idx.zero_()
    eng.key.zero_()
    return tok.clone()


def main(argv=None):
    """Time the batched prefill of a random prompt (CUDA events, best of 3 after a warm
    call); ``--profile`` adds torch's CUDA kernel table of one prefill."""
    import argparse
    import json

    from .config import SparkConfig, spark_x26_config
    from .model import DecodeEngine, SyntheticWeights
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", choices=["synthetic-4b", "spark-x26"], default="synthetic-4b")
    ap.add_argument("--tokens", type=int, default=2048)
    ap.add_argument("--profile", action="store_true")
    ap.add_argument("--gemm", choices=["q4", "bf16"], default="q4")
    args = ap.parse_args(argv)
    cfg = spark_x26_config() if args.model == "spark-x26" else SparkConfig()
    w = SyntheticWeights(cfg, device="cuda", seed=0)
    eng = DecodeEngine(w, max_seq_len=args.tokens + 64, num_blocks=(args.tokens + 64) // 128 + 8, use_graph=False)
    prompt = torch.randint(0, cfg.vocab_size, (args.tokens,), generator=torch.Generator().manual_seed(0),
                           dtype=torch.int32)
    eng.prefill_batched(prompt, gemm=args.gemm)
    torch.cuda.synchronize()
    best = None
    for _ in range(3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        eng.prefill_batched(prompt, gemm=args.gemm)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        best = ms if best is None else min(best, ms)
    print(json.dumps({"model": cfg.name, "tokens": args.tokens, "gemm": args.gemm, "ttft_ms": round(best, 3)}))
    if args.profile:
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            eng.prefill_batched(prompt, gemm=args.gemm)
            torch.cuda.synchronize()
        print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=12, max_name_column_width=70))


if __name__ == "__main__":
    main()
