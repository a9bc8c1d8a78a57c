"""GPU check of spark_attn_decode_noalloc, the attention entry point for callers that
cannot allocate device memory (its workspace is a static array inside the library).

It is called straight through the C ABI and must give exactly what the workspace-based
spark_attn_decode gives, on two calls in a row (the shared array keeps the previous
call's contents; the arrival counters must come back to zero).  This file is named to
be collected last; it also passes when run alone in a fresh process, where its first
call performs the once-per-device set-up.
"""
from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _dev_bf16(torch, a, device):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16)).view(torch.bfloat16).to(device)


def test_noalloc_attention_matches_workspace_entry_point(cuda, oracle):
    import torch
    from spark_b200 import _lib

    L = _lib.lib()
    P = ctypes.c_void_p
    nq, nkv, D, bs = 32, 8, 128, 128
    scale = ctypes.c_float(float(np.float32(1 / math.sqrt(D))))
    rng = np.random.default_rng(2024)
    stream = P(torch.cuda.current_stream().cuda_stream)
    for call, (ctx, splits) in enumerate([(3000, 48), (777, 16)]):
        nblk = (ctx + bs - 1) // bs
        kc = _dev_bf16(torch, oracle.f32_to_bf16(rng.standard_normal((2 * nblk, nkv, bs, D)).astype(np.float32)), cuda)
        vc = _dev_bf16(torch, oracle.f32_to_bf16(rng.standard_normal((2 * nblk, nkv, bs, D)).astype(np.float32)), cuda)
        table = torch.from_numpy(rng.permutation(2 * nblk)[:nblk].astype(np.int32)).to(cuda)
        q = _dev_bf16(torch, oracle.f32_to_bf16(rng.standard_normal((nq, D)).astype(np.float32)), cuda)
        pos = torch.tensor([ctx - 1], dtype=torch.int64, device=cuda)
        T = oracle.split_tokens(ctx, splits)
        # existing entry point with caller-owned workspace
        part_o = torch.empty((splits, nq, D), dtype=torch.float32, device=cuda)
        part_lse = torch.empty((splits, nq), dtype=torch.float32, device=cuda)
        counters = torch.zeros(nkv, dtype=torch.int32, device=cuda)
        ref = torch.empty((nq, D), dtype=torch.bfloat16, device=cuda)
        st = L.spark_attn_decode(P(q.data_ptr()), P(kc.data_ptr()), P(vc.data_ptr()), P(table.data_ptr()),
                                 P(pos.data_ptr()), None, nq, nkv, D, bs, splits, T, scale, P(part_o.data_ptr()),
                                 P(part_lse.data_ptr()), P(counters.data_ptr()), P(ref.data_ptr()), None, stream)
        assert st == 0
        # allocation-free entry point
        out = torch.full((nq, D), float("nan"), dtype=torch.bfloat16, device=cuda)
        err = torch.zeros(1, dtype=torch.int32, device=cuda)
        st = L.spark_attn_decode_noalloc(P(q.data_ptr()), P(kc.data_ptr()), P(vc.data_ptr()), P(table.data_ptr()),
                                         P(pos.data_ptr()), None, nq, nkv, D, bs, splits, T, scale,
                                         P(out.data_ptr()), P(err.data_ptr()), stream)
        assert st == 0, L.spark_status_string(st)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        # the attention tests hold this kernel to bit-exactness; so does this one
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), f"call {call}"
        assert not torch.isnan(out.float()).any()


def test_noalloc_attention_rejects_oversized_requests(cuda):
    from spark_b200 import _lib

    L = _lib.lib()
    fake = ctypes.c_void_p(0x1000)  # never dereferenced: the size check comes first
    st = L.spark_attn_decode_noalloc(fake, fake, fake, fake, fake, None, 32, 8, 128, 128, 65, 64,
                                     ctypes.c_float(0.1), fake, None, None)
    assert st == 5 and b"limit" in L.spark_status_string(st)
