"""The reference's benchmark modes on the B200 engine.

Mirrors hayate's ``benchmark.py`` (benchmark.py:168-431): the same three modes
-- single request (each request alone, latency per request), submit all
upfront (one ``generate_text`` over the whole set), staggered arrivals
(requests join a running engine at a fixed gap, latency from arrival to
completion) -- with the same summary columns (mean / p50 / p95 latency, gen
tok/s, total tok/s, where total counts prompt + generated tokens as
benchmark.py:187,228,296 do).  Prompts are uniform-random token ids of the
requested lengths (no tokenizer offline).  Two more modes cover the other
benchmark configurations: ``poisson`` (exponential inter-arrival gaps,
log-uniform prompts, chunked prefill mixed into decodes), ``replicas``
(requests spread over N GPU replicas by ``router.Router``) and ``shared_prefix``
(requests with a common 1024-token prefix, without and with the prefix cache).

``python -m hayate_b200.benchmark 10 [--repetitions 5] [--max-tokens 256]
[--seed 1337] [--arrival-gap-ms 25] [--min-prompt-tokens 160]
[--max-prompt-tokens 320] [--verbose] [--modes single,upfront,staggered]``
"""
from __future__ import annotations

import argparse
import json
import random
import time
from typing import Dict, List

import torch

from .config import EngineConfig
from .engine import Engine, Request
from . import workloads

DEFAULT_SEED = 1337
DEFAULT_MAX_TOKENS = 256
DEFAULT_REPETITIONS = 5
DEFAULT_ARRIVAL_GAP_MS = 25.0
DEFAULT_PROMPT_TOKENS_MIN = 160
DEFAULT_PROMPT_TOKENS_MAX = 320


def sync():
    if torch.cuda.is_available():
        torch.cuda.synchronize()


def percentile(values, pct):
    """Linear-interpolated percentile (the reference's definition, benchmark.py:73-86)."""
    if not values:
        return 0.0
    v = sorted(values)
    idx = (len(v) - 1) * pct / 100.0
    lo = int(idx)
    hi = min(lo + 1, len(v) - 1)
    w = idx - lo
    return v[lo] * (1 - w) + v[hi] * w


def make_requests(n, max_tokens, seed, lo, hi, vocab=workloads.VOCAB):
    rng = random.Random(seed)
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        L = rng.randint(lo, hi)
        out.append({"prompt": torch.randint(0, vocab, (L,), generator=g).tolist(),
                    "max_tokens": max_tokens})
    return out


def _result(latencies, elapsed, gen, total):
    return {"latencies": latencies, "elapsed": elapsed, "generated_tokens": gen,
            "total_tokens": total}


def bench_single(engine, reqs, reps):
    engine.generate_text(reqs[0]["prompt"], max_tokens=reqs[0]["max_tokens"])   # warm-up
    lat, gen, tot, el = [], 0, 0, 0.0
    for _ in range(reps):
        for r in reqs:
            sync()
            t0 = time.perf_counter()
            res = engine.generate_text(r["prompt"], max_tokens=r["max_tokens"])
            sync()
            dt = time.perf_counter() - t0
            lat.append(dt)
            el += dt
            gen += len(res.tokens)
            tot += len(r["prompt"]) + len(res.tokens)
    return _result(lat, el, gen, tot)


def bench_upfront(engine, reqs, reps):
    engine.generate_text([r["prompt"] for r in reqs[:2]], max_tokens=reqs[0]["max_tokens"])
    lat, gen, tot, el = [], 0, 0, 0.0
    ptoks = sum(len(r["prompt"]) for r in reqs)
    for _ in range(reps):
        sync()
        t0 = time.perf_counter()
        res = engine.generate_text([r["prompt"] for r in reqs], max_tokens=reqs[0]["max_tokens"])
        sync()
        dt = time.perf_counter() - t0
        res = res if isinstance(res, list) else [res]
        g = sum(len(x.tokens) for x in res)
        lat.append(dt)
        el += dt
        gen += g
        tot += ptoks + g
    return _result(lat, el, gen, tot)


def run_arrivals(engine, reqs, arrival_s: List[float]):
    """Requests join at their arrival times; latency = completion - arrival
    (benchmark.py:239-303)."""
    subs, done, meta = [], {}, {}
    nxt = 0
    sync()
    start = time.perf_counter()
    while nxt < len(reqs) or engine.current_batch or not engine.pool.empty():
        now = time.perf_counter() - start
        while nxt < len(reqs) and arrival_s[nxt] <= now:
            r = Request(id=engine.request_id, prompt=reqs[nxt]["prompt"],
                        max_tokens=reqs[nxt]["max_tokens"])
            engine.request_id += 1
            engine.add_request(r)
            subs.append(r)
            meta[r.id] = (time.perf_counter(), len(reqs[nxt]["prompt"]))
            nxt += 1
        stepped = engine.generate()
        for r in subs:
            if r.is_completed and r.id not in done:
                done[r.id] = time.perf_counter()
        if not stepped and nxt < len(reqs):
            wait = arrival_s[nxt] - (time.perf_counter() - start)
            if wait > 0:
                time.sleep(wait)
    sync()
    el = time.perf_counter() - start
    lat = [done[r.id] - meta[r.id][0] for r in subs]
    gen = sum(len(r.tokens) for r in subs)
    tot = sum(meta[r.id][1] + len(r.tokens) for r in subs)
    return _result(lat, el, gen, tot)


def bench_staggered(engine, reqs, reps, gap_ms):
    gaps = [i * gap_ms / 1000.0 for i in range(len(reqs))]
    run_arrivals(engine, reqs[:2], gaps[:2])
    out = _result([], 0.0, 0, 0)
    for _ in range(reps):
        r = run_arrivals(engine, reqs, gaps)
        out["latencies"] += r["latencies"]
        for k in ("elapsed", "generated_tokens", "total_tokens"):
            out[k] += r[k]
    return out


def bench_poisson(engine, seed, reps):
    """64 requests, exponential gaps of mean 20 ms, log-uniform prompts [128,2048],
    outputs U[128,512]."""
    ws = workloads.poisson(seed=seed)
    reqs = [{"prompt": w.prompt, "max_tokens": w.max_tokens} for w in ws]
    arr = [w.arrival_s for w in ws]
    run_arrivals(engine, reqs[:2], arr[:2])
    out = _result([], 0.0, 0, 0)
    for _ in range(reps):
        r = run_arrivals(engine, reqs, arr)
        out["latencies"] += r["latencies"]
        for k in ("elapsed", "generated_tokens", "total_tokens"):
            out[k] += r[k]
    return out


def bench_shared_prefix(n_requests, seed, reps, prefix_caching, prefix_len=1024, max_tokens=128):
    """Requests sharing a ``prefix_len``-token prefix (a common system prompt) with
    unique suffixes of U[16,128] tokens, all submitted at once, on an engine with
    or without the prefix cache.  The first request runs alone beforehand, as an
    earlier user of the same prefix would have."""
    rng = random.Random(seed)
    g = torch.Generator().manual_seed(seed)
    prefix = torch.randint(0, workloads.VOCAB, (prefix_len,), generator=g).tolist()
    reqs = [prefix + torch.randint(0, workloads.VOCAB, (rng.randint(16, 128),),
                                   generator=g).tolist() for _ in range(n_requests)]
    ecfg = default_engine_config(max_tokens, prefix_len + 128).with_(prefix_caching=prefix_caching)
    eng = Engine("Qwen/Qwen3-4B", engine_config=ecfg)
    eng.capture_graphs()
    eng.generate_text(reqs[0], max_tokens=max_tokens)
    out = _result([], 0.0, 0, 0)
    for _ in range(reps):
        sync()
        t0 = time.perf_counter()
        res = eng.generate_text(reqs, max_tokens=max_tokens)
        sync()
        dt = time.perf_counter() - t0
        out["latencies"].append(dt)
        out["elapsed"] += dt
        out["generated_tokens"] += sum(len(r.tokens) for r in res)
        out["total_tokens"] += sum(len(p) for p in reqs) + sum(len(r.tokens) for r in res)
    out["prompt_tokens_computed"] = eng.prompt_tokens_computed
    del eng
    torch.cuda.empty_cache()
    return out


def bench_replicas(n_gpus, seed, n_requests, engine_kwargs):
    """Requests U[512,4096] prompts, 256 tokens, spread over n_gpus replicas."""
    from .router import Router
    ws = workloads.replicas(seed=seed, n=n_requests)
    with Router(n_gpus, factory_kwargs=engine_kwargs) as router:
        while not all(router.ready):
            router.poll(0.5)
        t0 = time.perf_counter()
        for w in ws:
            router.submit(w.prompt, w.max_tokens)
        res = router.wait_all()
        el = time.perf_counter() - t0
    gen = sum(len(t) for t in res.values())
    tot = gen + sum(len(w.prompt) for w in ws)
    return _result([el], el, gen, tot)


def summarize(rows, verbose=False):
    print(f"\n  {'mode':<20} {'mean':>10} {'p50':>10} {'p95':>10} {'gen tok/s':>12} {'total tok/s':>12}")
    print(f"  {'-' * 20} {'-' * 10} {'-' * 10} {'-' * 10} {'-' * 12} {'-' * 12}")
    for title, r in rows:
        lat = r["latencies"] or [0.0]
        print(f"  {title:<20} {sum(lat) / len(lat):>9.3f}s {percentile(lat, 50):>9.3f}s "
              f"{percentile(lat, 95):>9.3f}s {r['generated_tokens'] / r['elapsed']:>11.2f} "
              f"{r['total_tokens'] / r['elapsed']:>11.2f}")


def replica_engine_config(share) -> EngineConfig:
    """Engine of one replica sized so that its whole share is admitted at once:
    a seat per request (at least 256) and every request's worst-case KV blocks
    (prompt + max_tokens) in the pool; 8192 tokens per step, 512-token chunks."""
    from .scheduler import blocks_for
    blocks = sum(blocks_for(len(w.prompt) + w.max_tokens, 16) for w in share) + 64
    longest = max(len(w.prompt) + w.max_tokens for w in share)
    return EngineConfig(max_num_seqs=max(256, len(share)), max_batched_tokens=8192,
                        prefill_chunk=512, num_kv_blocks=blocks, max_model_len=longest + 16,
                        cuda_graphs=True, ignore_eos=True)


def default_engine_config(max_tokens, max_prompt):
    return EngineConfig(max_num_seqs=256, max_batched_tokens=8192, prefill_chunk=512,
                        max_model_len=max_prompt + max_tokens + 16, ignore_eos=True)


def main(argv=None):
    ap = argparse.ArgumentParser(description="Benchmark the hayate_b200 engine.")
    ap.add_argument("n_requests", nargs="?", type=int, default=10)
    ap.add_argument("--repetitions", type=int, default=DEFAULT_REPETITIONS)
    ap.add_argument("--max-tokens", type=int, default=DEFAULT_MAX_TOKENS)
    ap.add_argument("--seed", type=int, default=DEFAULT_SEED)
    ap.add_argument("--arrival-gap-ms", type=float, default=DEFAULT_ARRIVAL_GAP_MS)
    ap.add_argument("--min-prompt-tokens", type=int, default=DEFAULT_PROMPT_TOKENS_MIN)
    ap.add_argument("--max-prompt-tokens", type=int, default=DEFAULT_PROMPT_TOKENS_MAX)
    ap.add_argument("--modes", default="single,upfront,staggered",
                    help="comma list of single, upfront, staggered, poisson, replicas, "
                         "shared_prefix")
    ap.add_argument("--gpus", type=int, default=1, help="replicas mode: GPU count")
    ap.add_argument("--replica-requests", type=int, default=2048)
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--json", default=None, help="write the results here")
    a = ap.parse_args(argv)
    if a.n_requests < 1 or a.repetitions < 1 or a.max_tokens < 1:
        raise ValueError("n_requests, repetitions and max_tokens must be at least 1")
    if a.min_prompt_tokens < 1 or a.min_prompt_tokens > a.max_prompt_tokens:
        raise ValueError("bad prompt token bounds")
    modes = [m.strip() for m in a.modes.split(",") if m.strip()]
    reqs = make_requests(a.n_requests, a.max_tokens, a.seed, a.min_prompt_tokens,
                         a.max_prompt_tokens)
    rows = []
    if any(m in modes for m in ("single", "upfront", "staggered", "poisson")):
        max_prompt = max(a.max_prompt_tokens, 2048 if "poisson" in modes else 0)
        eng = Engine("Qwen/Qwen3-4B", engine_config=default_engine_config(
            max(a.max_tokens, 512), max_prompt))
        if "single" in modes:
            rows.append(("single request", bench_single(eng, reqs, a.repetitions)))
        if "upfront" in modes:
            rows.append(("submit all upfront", bench_upfront(eng, reqs, a.repetitions)))
        if "staggered" in modes:
            rows.append(("staggered arrivals",
                         bench_staggered(eng, reqs, a.repetitions, a.arrival_gap_ms)))
        if "poisson" in modes:
            rows.append(("poisson arrivals", bench_poisson(eng, a.seed, a.repetitions)))
        del eng
        torch.cuda.empty_cache()
    if "shared_prefix" in modes:
        for on in (False, True):
            rows.append((f"shared prefix, cache {'on' if on else 'off'}",
                         bench_shared_prefix(64, a.seed, a.repetitions, on)))
    if "replicas" in modes:
        kw = {"engine_config": default_engine_config(256, 4096)}
        rows.append((f"replicas x{a.gpus}", bench_replicas(a.gpus, a.seed, a.replica_requests, kw)))
    summarize(rows, a.verbose)
    if a.json:
        with open(a.json, "w") as f:
            json.dump({t: {k: v for k, v in r.items()} for t, r in rows}, f)
    return rows


if __name__ == "__main__":
    main()
