"""Operator microbenchmarks of the hot-path kernels.

attention: the ragged attention case -- 256 decode sequences with contexts
log-uniform in [256,16384] plus 4 prefill chunks of 512 query tokens (prior
contexts 0, 512, 1536, 3584), 32 query / 8 KV heads, head_dim 128, bf16 Q/K/V
~ N(0,1), paged KV in 16-token blocks behind a randomly permuted block table,
one layer.  Its KV (~4 GB) is far larger than L2, so launches need no flush.

qk_norm_rope / kv_append / pack / argmax / add_rms_norm / silu_mul: the same
batch (2304 query tokens: 256 decode rows + 4 x 512 prefill rows) through the
fused QK-norm+RoPE+append kernel, the standalone KV append, the packing kernel,
the greedy argmax over the 256+4 sampled rows (vocab 151936), and the residual
add + RMSNorm (hidden 2560) and SiLU(gate)*up (9728) on its rows.  lm_head: the
LM head and greedy choice over the 256 decode rows (hidden 2560, vocab 151936),
the fused kernel against cuBLAS + argmax.  These inputs fit in L2, so each timed
launch is preceded by an L2 flush outside the timed window: a read of 256 MiB,
which evicts the op's data without leaving dirty lines whose write-back the
timed launch would pay.
``--tokens`` raises the token count of the append kernels (prefill-sized
batches).  Every op reports its algorithmic bytes; packing is latency-bound,
so its microseconds are the figure of merit.

``--stream`` times the row kernels as they run inside an engine step instead:
back to back, replayed from a CUDA graph, each launch on its own copy of the
inputs, with enough copies that together they are more than twice L2 (so every
launch reads its inputs from HBM); the figure is the graph's time over its
launches.  A single flushed launch also carries the launch and event overhead
(~10 us), which at prefill sizes is as long as the kernel.

``python -m hayate_b200.microbench [--op attention|qk_norm_rope|kv_append|pack|argmax|
lm_head|add_rms_norm|silu_mul|all]
[--iters N]`` prints one JSON line per op.
"""
from __future__ import annotations

import argparse
import json
import statistics

import numpy as np
import torch


def attention_micro_batch(n_decode: int = 256, prefill: bool = True, ctx_lo: int = 256,
                          ctx_hi: int = 16384, priors=None, seed: int = 0):
    """The ragged attention operator batch on the current device: 256 decode
    sequences with contexts log-uniform in [ctx_lo, ctx_hi] plus 512-token
    prefill chunks after ``priors`` (default 0, 512, 1536, 3584), 32 query / 8
    KV heads, bf16 Q and cache ~ N(0,1), one layer, 16-token blocks behind a
    randomly permuted block table.  Returns a dict of its tensors and shapes."""
    from hayate_b200.workloads import attn_micro
    w = attn_micro(seed=seed, n_decode=n_decode, lo=ctx_lo, hi=ctx_hi)
    if priors is not None:
        w.prefill_prior = list(priors)
    if not prefill:
        w.prefill_prior = []
    q_lens, kv_lens = w.q_lens(), w.seq_lens_k()
    S, T = len(q_lens), sum(q_lens)
    Hkv, Hq, D = 8, 32, 128
    nblk = [-(-k // 16) for k in kv_lens]
    NB = sum(nblk) + 64
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(seed)
    cache = torch.randn(1, NB, 2, Hkv, 16, D, device=dev, dtype=torch.bfloat16, generator=g)
    q = torch.randn(T, Hq, D, device=dev, dtype=torch.bfloat16, generator=g)
    perm = torch.randperm(NB, device=dev, generator=g).to(torch.int32)
    maxb = max(nblk)
    bt = torch.full((S, maxb), -1, dtype=torch.int32, device=dev)
    off = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[off:off + n]
        off += n
    cu = torch.tensor([0] + list(np.cumsum(q_lens)), dtype=torch.int32, device=dev)
    kv = torch.tensor(kv_lens, dtype=torch.int32, device=dev)
    return {"q": q, "cache": cache, "bt": bt, "cu": cu, "kv": kv, "S": S, "T": T,
            "q_lens": q_lens, "kv_lens": kv_lens, "nblk": nblk, "decode_seqs": len(w.decode_ctx),
            "prefill_chunks": len(w.prefill_prior)}


def attention_micro(iters: int = 20, n_decode: int = 256, prefill: bool = True,
                    ctx_lo: int = 256, ctx_hi: int = 16384, priors=None):
    """The ragged attention operator case: returns timing + algorithmic bytes.
    ``ctx_lo``/``ctx_hi`` bound the log-uniform decode contexts; ``priors`` (a
    list of prior context lengths, one 512-token prefill chunk each) replaces
    the operator case's four chunks."""
    from hayate_b200 import kernels as K
    b = attention_micro_batch(n_decode, prefill, ctx_lo, ctx_hi, priors)
    q, cache, bt, cu, kv, S, T = b["q"], b["cache"], b["bt"], b["cu"], b["kv"], b["S"], b["T"]
    q_lens, kv_lens, nblk = b["q_lens"], b["kv_lens"], b["nblk"]
    Hkv, Hq, D = 8, 32, 128
    dev = q.device
    out = torch.empty_like(q)
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
    for a, e in ev:
        a.record()
        launch()
        e.record()
    torch.cuda.synchronize()
    ms = [a.elapsed_time(e) for a, e in ev]
    if int(err.item()) != 0:
        raise RuntimeError(f"attention micro: device error {int(err.item())}")
    kv_bytes = sum(kv_lens) * Hkv * D * 2 * 2                  # K and V, read once
    qo_bytes = T * Hq * D * 2 * 2                             # q in, out
    bt_bytes = 4 * sum(nblk)
    pre_flops = sum(4 * Hq * D * (ql * (kl - ql) + ql * (ql + 1) / 2)
                    for ql, kl in zip(q_lens, kv_lens) if ql > 1)
    dec_bytes = sum(k * Hkv * D * 4 for ql, k in zip(q_lens, kv_lens) if ql == 1)
    del cache, b
    torch.cuda.empty_cache()
    return {"ms_mean": statistics.mean(ms), "ms_min": min(ms), "bytes": kv_bytes + qo_bytes + bt_bytes,
            "decode_kv_bytes": dec_bytes, "prefill_flops": pre_flops, "iters": iters,
            "decode_seqs": len([x for x in q_lens if x == 1]),
            "prefill_chunks": len([x for x in q_lens if x > 1])}


L2_FLUSH_BYTES = 256 << 20
L2_BYTES = 126 << 20


def _flusher():
    buf = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    return lambda: buf.sum()


def _time(launch, iters: int, flush: bool):
    """CUDA-event time of each launch (ms), after 3 warm-up launches; an L2
    flush precedes every timed launch when ``flush``."""
    flush_l2 = _flusher() if flush else None
    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    ms = []
    for _ in range(iters):
        if flush_l2 is not None:
            flush_l2()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        launch()
        b.record()
        b.synchronize()
        ms.append(a.elapsed_time(b))
    return ms


def _copies(set_bytes: int, cap: int = 16) -> int:
    """Input copies whose total is at least twice L2."""
    return max(2, min(cap, -(-2 * L2_BYTES // max(1, set_bytes))))


def _time_stream(launches, iters: int):
    """Per-launch time (ms) of ``launches`` (callables on disjoint buffers)
    replayed back to back from one CUDA graph, ``iters`` replays after 2 warm-up
    replays."""
    for f in launches:
        f()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for f in launches:
            f()
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    ms = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        b.synchronize()
        ms.append(a.elapsed_time(b) / len(launches))
    del g
    return ms


def _summary(op, ms, nbytes, **extra):
    mean = statistics.mean(ms)
    out = {"op": op, "ms_mean": mean, "ms_min": min(ms), "us_mean": mean * 1e3,
           "bytes": nbytes, "gbs": nbytes / (mean * 1e-3) / 1e9, "iters": len(ms)}
    out.update(extra)
    return out


def _batch_rows(n_decode: int, tokens: int):
    """(prior contexts, q_lens) of the operator batch: decode rows of the
    attention case, then prefill chunks of 512 up to ``tokens`` query tokens."""
    from hayate_b200.workloads import attn_micro
    w = attn_micro(seed=0, n_decode=n_decode)
    prior = list(w.decode_ctx)
    q = [1] * len(prior)
    pre = [0, 512, 1536, 3584]
    k = 0
    while sum(q) + 512 <= tokens:
        prior.append(pre[k % 4] + 4096 * ((k // 4) % 8))   # positions stay < 32768 + 512
        q.append(512)
        k += 1
    return prior, q


def append_micro(iters: int = 20, n_decode: int = 256, tokens: int = 2304, fused: bool = True,
                 stream: bool = False):
    """Fused QK-RMSNorm + RoPE + paged KV append (``fused``) or the standalone
    KV append, over the tokens of the operator batch (``stream``: see the
    module docstring)."""
    from hayate_b200 import kernels as K
    prior, q_lens = _batch_rows(n_decode, tokens)
    T = sum(q_lens)
    Hq, Hkv, D = 32, 8, 128
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    # only the blocks the step writes exist; they sit at random places in the cache
    spans = [(p // 16, (p + q - 1) // 16) for p, q in zip(prior, q_lens)]
    NB = sum(b - a + 1 for a, b in spans) + 64
    cache = torch.zeros(NB, 2, Hkv, 16, D, device=dev, dtype=torch.bfloat16)
    perm = torch.randperm(NB, device=dev, generator=g).tolist()
    slots, pos, off = [], [], 0
    for (p, q), (a, b) in zip(zip(prior, q_lens), spans):
        pos += list(range(p, p + q))
        slots += [perm[off + t // 16 - a] * 16 + t % 16 for t in range(p, p + q)]
        off += b - a + 1
    smap = torch.tensor(slots, dtype=torch.int32, device=dev)
    positions = torch.tensor(pos, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    if fused:
        max_pos = 40960
        qn = torch.ones(D, device=dev, dtype=torch.bfloat16)
        ang = torch.rand(max_pos, 64, device=dev, generator=g) * 6.28
        cos, sin = torch.cos(ang), torch.sin(ang)
        # qkv row in, q out, K and V into the cache, position + slot, cos + sin rows
        nbytes = T * ((Hq + 2 * Hkv) * D * 2 + Hq * D * 2 + 2 * Hkv * D * 2 + 8 + 2 * 64 * 4)
        op = "qk_norm_rope"

        def make(c):
            qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=dev, dtype=torch.bfloat16,
                              generator=g)
            q_out = torch.empty(T, Hq, D, device=dev, dtype=torch.bfloat16)
            return lambda: K.qk_norm_rope(qkv, Hq, Hkv, positions, qn, qn, cos, sin, 1e-6,
                                          q_out=q_out, kv_cache_layer=c, slot_mapping=smap,
                                          num_blocks=NB, err=err)
    else:
        nbytes = T * (2 * 2 * Hkv * D * 2 + 4)        # K and V read and written, slot
        op = "kv_append"

        def make(c):
            k = torch.randn(T, Hkv, D, device=dev, dtype=torch.bfloat16, generator=g)
            v = torch.randn(T, Hkv, D, device=dev, dtype=torch.bfloat16, generator=g)
            return lambda: K.kv_append(k, v, smap, c, NB, err=err)
    if stream:
        ms = _time_stream([make(cache if i == 0 else torch.zeros_like(cache))
                           for i in range(_copies(nbytes))], iters)
    else:
        ms = _time(make(cache), iters, flush=True)
    if int(err.item()) != 0:
        raise RuntimeError(f"{op} micro: device error {int(err.item())}")
    return _summary(op, ms, nbytes, tokens=T)


def pack_micro(iters: int = 20, n_decode: int = 256, tokens: int = 2304):
    """Packing of the operator batch: every sequence has its prior context
    cached (its blocks owned), the step adds q_len tokens and allocates the
    blocks they start."""
    from hayate_b200 import kernels as K
    prior, q_lens = _batch_rows(n_decode, tokens)
    S, T = len(prior), sum(q_lens)
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    max_reqs = S + 1
    tok_pitch = max(p + q for p, q in zip(prior, q_lens))
    bt_pitch = -(-tok_pitch // 16)
    have = [-(-p // 16) for p in prior]
    need = [-(-(p + q) // 16) - h for p, q, h in zip(prior, q_lens, have)]
    NB = sum(have) + sum(need) + 64
    req_tokens = torch.randint(0, 151936, (max_reqs, tok_pitch), device=dev,
                               dtype=torch.int32, generator=g)
    bt0 = torch.full((max_reqs, bt_pitch), -1, dtype=torch.int32, device=dev)
    perm = torch.randperm(NB, device=dev, generator=g).to(torch.int32)
    off = 0
    for i, h in enumerate(have):
        bt0[i, :h] = perm[off:off + h]
        off += h
    free0 = torch.full((NB,), -1, dtype=torch.int32, device=dev)
    free0[:NB - off] = perm[off:]
    nblk0 = torch.tensor(have + [0], dtype=torch.int32, device=dev)
    top0 = torch.tensor([NB - off], dtype=torch.int32, device=dev)
    sched = torch.tensor([list(range(S)), prior, q_lens, [1] * S], dtype=torch.int32,
                         device=dev).flatten().contiguous()
    bt, nblk, free, top = bt0.clone(), nblk0.clone(), free0.clone(), top0.clone()
    ids, positions, smap = (torch.empty(T, dtype=torch.int32, device=dev) for _ in range(3))
    cu_q, kv_lens = (torch.empty(S + 1, dtype=torch.int32, device=dev) for _ in range(2))
    rows, seqs = (torch.empty(S, dtype=torch.int32, device=dev) for _ in range(2))
    err = torch.zeros(1, dtype=torch.int32, device=dev)

    def launch():
        K.pack_batch(sched, S, T, req_tokens, bt, nblk, free, top, ids, positions, smap,
                     cu_q, kv_lens, rows, seqs, err)

    def reset():
        bt.copy_(bt0); nblk.copy_(nblk0); free.copy_(free0); top.copy_(top0)

    ms = []
    flush_l2 = _flusher()
    for i in range(iters + 3):
        reset()
        flush_l2()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        launch()
        b.record()
        b.synchronize()
        if i >= 3:
            ms.append(a.elapsed_time(b))
    if int(err.item()) != 0:
        raise RuntimeError(f"pack micro: device error {int(err.item())}")
    # reads: schedule, owned-block counts, token ids, block-table entries, popped
    # stack entries; writes: ids, positions, slots, cu_q, seq_lens_k, sample rows,
    # new block-table entries, counts
    nbytes = 4 * (4 * S + S + T + T + sum(need)) + 4 * (3 * T + (S + 1) + S + 2 * S + sum(need) + S)
    return _summary("pack", ms, nbytes, seqs=S, tokens=T, new_blocks=sum(need))


def argmax_micro(iters: int = 20, rows: int = 260, vocab: int = 151936, stream: bool = False):
    """Greedy argmax over ``rows`` bf16 logit rows (the sampled rows of the
    operator batch; ``stream``: see the module docstring)."""
    from hayate_b200 import kernels as K
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    nbytes = rows * vocab * 2 + rows * 4
    sets = []
    for _ in range(_copies(nbytes) if stream else 1):
        logits = torch.randn(rows, vocab, device=dev, dtype=torch.bfloat16, generator=g)
        sets.append((logits, torch.empty(rows, dtype=torch.int32, device=dev)))
    launches = [(lambda lo=lo, o=o: K.argmax(lo, o)) for lo, o in sets]
    ms = _time_stream(launches, iters) if stream else _time(launches[0], iters, flush=True)
    for logits, out in sets:
        if not torch.equal(out.long(), logits.argmax(dim=1)):
            raise RuntimeError("argmax micro: result differs from torch.argmax")
    return _summary("argmax", ms, nbytes, rows=rows, stream=stream)


def lm_head_micro(iters: int = 20, rows: int = 256, vocab: int = 151936, hidden: int = 2560):
    """The LM head and the greedy choice over ``rows`` sampled rows at Qwen3-4B
    sizes: ``hy_lm_head_argmax`` (one kernel, logits never written) against the
    cuBLAS GEMM + ``hy_argmax`` pair it replaces.  The weights (778 MB) exceed
    L2, so launches need no flush between them.  ``bytes`` is the fused
    kernel's algorithmic traffic: W and x read once, the tokens written."""
    import torch.nn.functional as F
    from hayate_b200 import kernels as K
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    w = torch.randn(vocab, hidden, device=dev, dtype=torch.bfloat16, generator=g) * 0.02
    x = torch.randn(rows, hidden, device=dev, dtype=torch.bfloat16, generator=g)
    ws = torch.zeros(K.lm_head_argmax_workspace_size(), dtype=torch.uint8, device=dev)
    out_f = torch.empty(rows, dtype=torch.int32, device=dev)
    out_u = torch.empty(rows, dtype=torch.int32, device=dev)
    ms_f = _time(lambda: K.lm_head_argmax(x, w, out_f, ws), iters, flush=False)
    ms_u = _time(lambda: K.argmax(F.linear(x, w), out_u), iters, flush=False)
    mism = int((out_f != out_u).sum().item())
    nbytes = vocab * hidden * 2 + rows * hidden * 2 + rows * 4
    r = _summary("lm_head", ms_f, nbytes, rows=rows, vocab=vocab, hidden=hidden)
    r["tflops"] = 2.0 * rows * vocab * hidden / (r["ms_mean"] * 1e-3) / 1e12
    r["unfused_ms_mean"] = statistics.mean(ms_u)
    r["token_mismatches_vs_unfused"] = mism
    return r


def rowwise_micro(op: str, iters: int = 20, rows: int = 2304, hidden: int = 2560,
                  inter: int = 9728, stream: bool = False):
    """Residual add + RMSNorm over [rows][hidden] (``add_rms_norm``) or SiLU(gate) * up
    over [rows][2 inter] (``silu_mul``), bf16, Qwen3-4B widths (``stream``: see
    the module docstring)."""
    from hayate_b200 import kernels as K
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    if op == "add_rms_norm":
        nbytes = rows * hidden * 2 * 4 + hidden * 2            # x, delta in; x, y out; weights
        w = torch.ones(hidden, device=dev, dtype=torch.bfloat16)

        def make():
            x = torch.randn(rows, hidden, device=dev, dtype=torch.bfloat16, generator=g)
            d = torch.randn(rows, hidden, device=dev, dtype=torch.bfloat16, generator=g)
            y = torch.empty_like(x)
            return lambda: K.add_rms_norm(x, w, 1e-6, delta=d, out=y)
    else:
        nbytes = rows * inter * 2 * 3                           # gate, up in; product out

        def make():
            gu = torch.randn(rows, 2 * inter, device=dev, dtype=torch.bfloat16, generator=g)
            y = torch.empty(rows, inter, device=dev, dtype=torch.bfloat16)
            return lambda: K.silu_mul(gu, y)
    if stream:
        ms = _time_stream([make() for _ in range(_copies(nbytes))], iters)
    else:
        ms = _time(make(), iters, flush=True)
    return _summary(op, ms, nbytes, rows=rows, stream=stream)


OPS = ("attention", "qk_norm_rope", "kv_append", "pack", "argmax", "lm_head", "add_rms_norm",
       "silu_mul")


def run_op(op: str, iters: int, n_decode: int = 256, prefill: bool = True, tokens: int = 2304,
           ctx_lo: int = 256, ctx_hi: int = 16384, priors=None, stream: bool = False):
    if op == "attention":
        r = attention_micro(iters, n_decode, prefill, ctx_lo, ctx_hi, priors)
        r["op"] = op
        r["gbs"] = r["bytes"] / (r["ms_mean"] * 1e-3) / 1e9
        r["prefill_tflops"] = r["prefill_flops"] / (r["ms_mean"] * 1e-3) / 1e12
        return r
    if op in ("qk_norm_rope", "kv_append"):
        r = append_micro(iters, n_decode, tokens, fused=op == "qk_norm_rope", stream=stream)
        r["stream"] = stream
        return r
    if op == "pack":
        return pack_micro(iters, n_decode, tokens)
    if op == "argmax":
        return argmax_micro(iters, rows=max(1, n_decode + max(0, tokens - n_decode) // 512),
                            stream=stream)
    if op == "lm_head":
        return lm_head_micro(iters, rows=max(1, n_decode))
    if op in ("add_rms_norm", "silu_mul"):
        return rowwise_micro(op, iters, rows=max(1, tokens), stream=stream)
    raise ValueError(f"unknown op {op!r}; one of {OPS} or 'all'")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", default="attention", help="one of " + ", ".join(OPS) + ", or all")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--decode", type=int, default=256,
                    help="decode sequences (fewer: a smaller case for profiling)")
    ap.add_argument("--no-prefill", action="store_true", help="attention: decode sequences only")
    ap.add_argument("--tokens", type=int, default=2304,
                    help="query tokens of the batch for the append, pack and argmax ops")
    ap.add_argument("--ctx-lo", type=int, default=256, help="attention: shortest decode context")
    ap.add_argument("--ctx-hi", type=int, default=16384, help="attention: longest decode context")
    ap.add_argument("--priors", default=None,
                    help="attention: comma-separated prior lengths, one 512-token prefill "
                         "chunk each (default: the operator case's 0,512,1536,3584)")
    ap.add_argument("--stream", action="store_true",
                    help="row kernels: graph-replayed back-to-back launches over input "
                         "copies larger than L2, instead of single flushed launches")
    a = ap.parse_args()
    priors = None if a.priors is None else [int(x) for x in a.priors.split(",") if x]
    torch.cuda.set_device(0)
    for op in (OPS if a.op == "all" else (a.op,)):
        print(json.dumps(run_op(op, a.iters, a.decode, not a.no_prefill, a.tokens, a.ctx_lo,
                                a.ctx_hi, priors, a.stream)), flush=True)


if __name__ == "__main__":
    main()
