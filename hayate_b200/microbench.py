"""Operator microbenchmark of the varlen paged attention kernel.

The ragged attention case: 256 decode sequences with contexts log-uniform in
[256,16384] plus 4 prefill chunks of 512 query tokens (prior contexts 0, 512,
1536, 3584), 32 query / 8 KV heads, head_dim 128, bf16 Q/K/V ~ N(0,1), paged KV
in 16-token blocks behind a randomly permuted block table, one layer.  The KV
of this case (~4 GB) is far larger than L2, so launches need no L2 flush.

``python -m hayate_b200.microbench [--iters N]`` prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import statistics

import numpy as np
import torch


def attention_micro(iters: int = 20, n_decode: int = 256, prefill: bool = True):
    """The ragged attention operator case: returns timing + algorithmic bytes."""
    from hayate_b200 import kernels as K
    from hayate_b200.workloads import attn_micro
    w = attn_micro(seed=0, n_decode=n_decode)
    if not prefill:
        w.prefill_prior = []
    q_lens, kv_lens = w.q_lens(), w.seq_lens_k()
    S, T = len(q_lens), sum(q_lens)
    Hkv, Hq, D = 8, 32, 128
    nblk = [-(-k // 16) for k in kv_lens]
    NB = sum(nblk) + 64
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    cache = torch.randn(1, NB, 2, Hkv, 16, D, device=dev, dtype=torch.bfloat16, generator=g)
    q = torch.randn(T, Hq, D, device=dev, dtype=torch.bfloat16, generator=g)
    out = torch.empty_like(q)
    perm = torch.randperm(NB, device=dev, generator=g).to(torch.int32)
    maxb = max(nblk)
    bt = torch.full((S, maxb), -1, dtype=torch.int32, device=dev)
    off = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[off:off + n]
        off += n
    cu = torch.tensor([0] + list(np.cumsum(q_lens)), dtype=torch.int32, device=dev)
    kv = torch.tensor(kv_lens, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = torch.zeros(K.attention_workspace_size(S, T, Hkv), dtype=torch.uint8, device=dev)
    K.attention_plan(cu, kv, S, Hkv, S, T, ws, err)

    def launch():
        K.varlen_attention(q, out, cache, 0, bt, cu, kv, S, S, T, ws, err=err)

    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(iters)]
    for a, b in ev:
        a.record()
        launch()
        b.record()
    torch.cuda.synchronize()
    ms = [a.elapsed_time(b) for a, b in ev]
    if int(err.item()) != 0:
        raise RuntimeError(f"attention micro: device error {int(err.item())}")
    kv_bytes = sum(kv_lens) * Hkv * D * 2 * 2                  # K and V, read once
    qo_bytes = T * Hq * D * 2 * 2                             # q in, out
    bt_bytes = 4 * sum(nblk)
    pre_flops = sum(4 * Hq * D * (ql * (kl - ql) + ql * (ql + 1) / 2)
                    for ql, kl in zip(q_lens, kv_lens) if ql > 1)
    dec_bytes = sum(k * Hkv * D * 4 for ql, k in zip(q_lens, kv_lens) if ql == 1)
    del cache
    torch.cuda.empty_cache()
    return {"ms_mean": statistics.mean(ms), "ms_min": min(ms), "bytes": kv_bytes + qo_bytes + bt_bytes,
            "decode_kv_bytes": dec_bytes, "prefill_flops": pre_flops, "iters": iters,
            "decode_seqs": len(w.decode_ctx), "prefill_chunks": len(w.prefill_prior)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--decode", type=int, default=256,
                    help="decode sequences (fewer: a smaller case for profiling)")
    ap.add_argument("--no-prefill", action="store_true", help="decode sequences only")
    a = ap.parse_args()
    torch.cuda.set_device(0)
    r = attention_micro(a.iters, a.decode, not a.no_prefill)
    r["gbs"] = r["bytes"] / (r["ms_mean"] * 1e-3) / 1e9
    print(json.dumps(r))


if __name__ == "__main__":
    main()
