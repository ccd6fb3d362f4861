"""Shared builders for the GPU parity tests."""
from __future__ import annotations

from typing import List, Sequence, Tuple

import torch

from oracle import reference as R

BLOCK = 16
D = 128


def random_paged_batch(q_lens: Sequence[int], kv_lens: Sequence[int], kv_heads: int,
                       dtype=torch.bfloat16, layers: int = 2, layer: int = 1, seed: int = 0,
                       spare_blocks: int = 7, device="cuda"):
    """A random KV cache with a randomly permuted block table per sequence.

    Returns dict with q (T, Hq, D), cache [layers][NB][2][Hkv][16][D], block
    table (S, max_blocks), cu_seqlens_q, seq_lens_k, and per-sequence contiguous
    K/V contexts (L_i, Hkv, D) gathered from ``layer``.
    """
    g = torch.Generator(device="cpu").manual_seed(seed)
    S = len(q_lens)
    nblk = [-(-kv // BLOCK) for kv in kv_lens]
    NB = sum(nblk) + spare_blocks
    maxb = max(max(nblk), 1)
    perm = torch.randperm(NB, generator=g)
    bt = torch.full((S, maxb), -1, dtype=torch.int32)
    off = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[off:off + n].to(torch.int32)
        off += n
    Hq = 4 * kv_heads
    cache = torch.randn(layers, NB, 2, kv_heads, BLOCK, D, generator=g).to(dtype)
    T = sum(q_lens)
    q = torch.randn(T, Hq, D, generator=g).to(dtype)
    cu = [0]
    for ql in q_lens:
        cu.append(cu[-1] + ql)
    ctx_k, ctx_v = [], []
    for i in range(S):
        blocks = cache[layer, bt[i, :nblk[i]].long()]            # (n, 2, Hkv, 16, D)
        k = blocks[:, 0].permute(0, 2, 1, 3).reshape(-1, kv_heads, D)[:kv_lens[i]]
        v = blocks[:, 1].permute(0, 2, 1, 3).reshape(-1, kv_heads, D)[:kv_lens[i]]
        ctx_k.append(k)
        ctx_v.append(v)
    return {
        "q": q.to(device), "cache": cache.to(device), "bt": bt.to(device),
        "cu": torch.tensor(cu, dtype=torch.int32, device=device),
        "kv": torch.tensor(list(kv_lens), dtype=torch.int32, device=device),
        "cu_list": cu, "ctx_k": [k.to(device) for k in ctx_k],
        "ctx_v": [v.to(device) for v in ctx_v], "S": S, "T": T, "layer": layer,
    }


def reference_attention(b) -> torch.Tensor:
    """fp32 reference (plain PyTorch SDPA with the reference's causal mask)."""
    return R.varlen_attention(b["q"], b["cu_list"], b["ctx_k"], b["ctx_v"])
