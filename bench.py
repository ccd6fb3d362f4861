"""Throughput benchmark of the B200 continuous-batching engine (one JSON line).

``python bench.py [--gpus N] [--steps K] [--warmup W] [--impl hayate|reference]``

Workload: the request-level data-parallel configuration the output-tok/s metric
is quoted on -- N x 256 requests, prompt lengths U[512,4096] (uniform-random
token ids), 256 greedy tokens each (fixed length, eos ignored), Qwen3-4B
architecture in bf16 with random N(0,0.02) weights.  The request set is split
over the N GPUs by the router's least-outstanding-work rule
(``router.least_work_assignment``), computed identically on every rank; each
rank is an independent engine replica on its own GPU (no collective on the
data path).  At N=8 the set is the 2048-request configuration; at N=1 it is the
256-request load one of its replicas carries.

A *step* is one complete run of the rank's share through the engine: every
request submitted at once, continuous batching (512-token prefill chunks mixed
into decode steps, paged KV) until all finish.  ``value`` is total output
tokens of all ranks over the slowest rank's device time; ``e2e`` is the same
metric through ``Engine.generate_text`` with host token lists in and out.

The line also carries the ragged-attention roofline (the operator case of 256
decode sequences with contexts log-uniform in [256,16384] plus 4 prefill
chunks of 512 tokens, one layer, paged KV in 16-token blocks), the 10-request
"submit all upfront" run (prompts U[64,512]) as a secondary figure, and, at
N=1, a CPU baseline: the reference algorithm (``oracle.reference``) timed on
this host's cores.  ``--impl reference`` times only that CPU path.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

PER_GPU = 256                      # requests per replica
MAX_TOKENS = 256
PROMPT_LO, PROMPT_HI = 512, 4096
WORKLOAD = ("replica share of N x 256 requests (the 2048-request set at N=8), prompt lengths "
            "U[512,4096], uniform-random ids, 256 greedy tokens each (eos ignored), split over "
            "the N GPUs by least outstanding work (prompt + max_tokens), every request of a "
            "share submitted at once; Qwen3-4B arch (36 layers, hidden 2560, 32/8 heads, "
            "head_dim 128, MLP 9728, vocab 151936) bf16")
WEIGHTS = ("random-init N(0,0.02) drawn on the GPU (torch.cuda generator, seed 0); the parity "
           "fixtures use the CPU recipe of the same distribution, and throughput does not "
           "depend on the values")
REF_BATCH = 20                     # the reference engine's MAX_BATCH_SIZE (engine.py:13)
PEAKS_FILE = os.path.join(REPO, "MEASURED_PEAKS.json")
FALLBACK_HBM_GBS = 6650.0


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ---------------------------------------------------------------------- dist
class stdout_to_stderr:
    """File descriptor 1 points at stderr inside the block (output of native
    libraries included)."""

    def __enter__(self):
        sys.stdout.flush()
        self.saved = os.dup(1)
        os.dup2(2, 1)
        return self

    def __exit__(self, *exc):
        sys.stdout.flush()
        os.dup2(self.saved, 1)
        os.close(self.saved)
        return False


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        # the communicator is created here and by the first collective; NCCL may
        # print its version on stdout then, which must carry only the JSON line
        with stdout_to_stderr():
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                    device_id=torch.device("cuda", local))
            barrier(world, local)
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world, local):
    if world > 1:
        import torch.distributed as dist
        if dist.get_backend() == "nccl":
            dist.barrier(device_ids=[local])
        else:
            dist.barrier()


def _reduce(x: float, world: int, op: str) -> float:
    """All-reduce one number over the ranks (NCCL on GPUs, gloo on CPU)."""
    if world == 1:
        return x
    import torch.distributed as dist
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=getattr(dist.ReduceOp, op))
    return float(t.item())


def max_over_ranks(x: float, world: int) -> float:
    return _reduce(x, world, "MAX")


def sum_over_ranks(x: float, world: int) -> float:
    return _reduce(x, world, "SUM")


# ---------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampled every 200 ms while the timed region runs."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.p = None
        try:
            uuid = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
            self.p = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", uuid], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
        except Exception:                                   # noqa: BLE001
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            out, _ = self.p.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.p.kill()
            out, _ = self.p.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------- engine arm
def rank_share(world: int, rank: int, seed: int = 0):
    """This rank's requests of the world x 256 request set (least outstanding
    work, the router's rule for requests that arrive together)."""
    from hayate_b200.workloads import replica_share
    return replica_share(world, rank, seed, PER_GPU)


def make_engine(device, share):
    """An engine sized so the whole share is admitted at once (every request's
    worst-case KV blocks reserved)."""
    from hayate_b200.benchmark import replica_engine_config
    from hayate_b200.engine import Engine
    return Engine("Qwen/Qwen3-4B", engine_config=replica_engine_config(share),
                  dtype=torch.bfloat16, weights="device", seed=0, device=device)


def run_workload(eng, prompts, max_tokens):
    reqs = eng.generate_text(prompts, max_tokens=max_tokens)
    reqs = reqs if isinstance(reqs, list) else [reqs]
    return sum(len(r.tokens) for r in reqs)


def timed(eng, fn, steps):
    """CUDA-event time (ms) of `steps` calls of fn on the engine's stream."""
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    start.record()
    toks = 0
    for _ in range(steps):
        toks += fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end), toks, (time.perf_counter() - w0) * 1e3


def read_peaks():
    try:
        with open(PEAKS_FILE) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:                                        # noqa: BLE001
        return FALLBACK_HBM_GBS, "fallback"


def profile_traffic():
    """DRAM bytes per launch of the attention kernel from the committed ncu summary."""
    path = os.path.join(REPO, "profiles", "varlen_attention_micro.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1].strip()))
    except OSError:
        pass
    return None


# ---------------------------------------------------------------------- CPU arm
CPU_SAMPLE = ("decode steps of the reference step loop restated on CPU (oracle/reference.py, "
              "engine.py:184-217) over its full batch of 20 requests (MAX_BATCH_SIZE) taken from "
              "the rank-0 share of this workload, bf16, their caches pre-filled with random "
              "values at their prompt lengths (a decode step's cost does not depend on them); "
              "prefill is not timed -- it is ~90% of this workload's tokens, so the CPU figure "
              "is an upper bound on the reference's throughput here")


def cpu_reference_decode(steps: int, warmup: int, seed: int = 0):
    """The reference step loop (oracle.reference.RefEngine) on this host's CPU
    cores: decode steps of a 20-request batch of the workload.  Returns
    (output tok/s, seconds per step, threads)."""
    from hayate_b200.config import QWEN3_4B as cfg
    from oracle import reference as R
    from hayate_b200 import weights as Wt
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(seed)

    def rnd(*shape):
        return (torch.randn(*shape, generator=g, dtype=torch.float32) * 0.02).to(torch.bfloat16)
    # the seed-0 weights of the parity fixtures, filled block-parallel
    Wr = R.RefWeights.from_host(Wt.exact_seeded(cfg, seed), torch.bfloat16)
    eng = R.RefEngine(Wr)
    batch = rank_share(1, 0, seed)[:REF_BATCH]
    for sr in batch:
        r = eng.add(sr.prompt, 10 ** 6)
        L = len(sr.prompt)
        r.k = rnd(cfg.num_layers, cfg.num_kv_heads, L, cfg.head_dim)
        r.v = rnd(cfg.num_layers, cfg.num_kv_heads, L, cfg.head_dim)
        r.cache_pos, r.is_prefill, r.tokens = L, False, [int(sr.prompt[-1])]
    for _ in range(warmup):
        eng.step()
    t0 = time.perf_counter()
    for _ in range(steps):
        eng.step()
    dt = (time.perf_counter() - t0) / steps
    return len(batch) / dt, dt, threads


def reference_arm(args, world, rank):
    if rank != 0:
        return
    tok_s, dt, threads = cpu_reference_decode(args.steps, args.warmup)
    line = {
        "impl": "reference", "metric": "total output tok/s", "value": tok_s, "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "requests_per_gpu": PER_GPU, "max_tokens": MAX_TOKENS,
                   "step": "one decode step of the reference engine over 20 requests",
                   "left_out": "prefill (not timed on the CPU)"},
        "cpu_baseline": {"value": tok_s, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": CPU_SAMPLE},
        "e2e": {"value": tok_s, "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------- main
E2E_RUNS = 3        # end-to-end runs (host lists in and out), after the device-resident ones


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="hayate", choices=["hayate", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--attn-iters", type=int, default=20)
    args = ap.parse_args()
    if args.warmup < 3:
        log("warmup raised to 3 (timing rule)")
        args.warmup = 3
    world, rank, local = dist_setup()
    if args.impl == "reference":
        reference_arm(args, world, rank)
        return
    from hayate_b200.workloads import upfront

    device = torch.device("cuda", local)
    share = rank_share(world, rank)
    eng = make_engine(device, share)
    eng.capture_graphs()                       # every decode bucket, before any timing
    host_prompts = [w.prompt for w in share]
    dev_prompts = [torch.tensor(p, dtype=torch.int32, device=device) for p in host_prompts]
    prompt_tokens = sum(len(p) for p in host_prompts)

    def device_run():
        return run_workload(eng, dev_prompts, MAX_TOKENS)

    def e2e_run():
        return run_workload(eng, host_prompts, MAX_TOKENS)

    for _ in range(args.warmup):
        device_run()
    e2e_run()
    barrier(world, local)
    launches0 = eng.runner.kernel_launches
    clk = ClockSampler(local)
    ms, toks, wall_ms = timed(eng, device_run, args.steps)
    clocks = clk.stop()
    launches = eng.runner.kernel_launches - launches0
    barrier(world, local)
    ms_max = max_over_ranks(ms, world)
    toks_all = sum_over_ranks(toks, world)

    e2e_steps = max(1, min(args.steps, E2E_RUNS))
    h0, d0 = eng.h2d_bytes, eng.d2h_bytes
    barrier(world, local)
    ems, etoks, ewall = timed(eng, e2e_run, e2e_steps)
    barrier(world, local)
    ems_max = max_over_ranks(ems, world)
    etoks_all = sum_over_ranks(etoks, world)
    h2d = (eng.h2d_bytes - h0) / e2e_steps
    d2h = (eng.d2h_bytes - d0) / e2e_steps

    # secondary: the 10-request "submit all upfront" run on the same engine
    c2 = [torch.tensor(r.prompt, dtype=torch.int32, device=device) for r in upfront(seed=rank)]
    run_workload(eng, c2, 256)
    c2_ms, c2_toks, _ = timed(eng, lambda: run_workload(eng, c2, 256), 3)
    err = eng.check_device_errors()
    if err:
        raise RuntimeError(f"device error word {err}")
    c2_line = {"workload": "10 requests, prompts U[64,512], 256 tokens each, all at once",
               "value": c2_toks / (c2_ms * 1e-3), "unit": "tok/s", "ms_per_run": c2_ms / 3,
               "runs": 3}

    # ragged-attention roofline (every rank runs it; rank 0 reports)
    del eng
    torch.cuda.empty_cache()
    from hayate_b200.microbench import attention_micro
    am = attention_micro(args.attn_iters)
    peak, peak_kind = read_peaks()
    achieved = am["bytes"] / (am["ms_mean"] * 1e-3) / 1e9

    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        tok_s, dt, threads = cpu_reference_decode(steps=3, warmup=1)
        cpu = {"value": tok_s, "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": "3 " + CPU_SAMPLE + " (after 1 warm-up step)"}
    if rank == 0:
        emit_line(args, world, toks_all, ms_max, wall_ms, etoks_all, ems_max, e2e_steps, h2d, d2h,
                  launches, am, achieved, peak, peak_kind, cpu, clocks, c2_line,
                  len(share), prompt_tokens)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def emit_line(args, world, toks_all, ms_max, wall_ms, etoks_all, ems_max, e2e_steps, h2d, d2h,
              launches, am, achieved, peak, peak_kind, cpu, clocks, c2_line, n_share,
              prompt_tokens):
    line = {
        "metric": "total output tok/s", "value": toks_all / (ms_max * 1e-3), "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (uniform-random token ids, random-init weights)",
        "config": {"workload": WORKLOAD, "weights": WEIGHTS, "requests_per_gpu": PER_GPU,
                   "requests_rank0": n_share, "prompt_tokens_rank0": prompt_tokens,
                   "max_tokens": MAX_TOKENS,
                   "parallelism": f"request-level replicas x{world} (no collective on the data path)",
                   "engine": "max_num_seqs 256, 8192 tokens per step, 512-token prefill chunks, "
                             "16-token KV blocks, CUDA-graph decode steps",
                   "step": "one full run of the rank's share (prefill + 256 decode tokens each)",
                   "l2": "no flush: every engine step streams 8 GB of weights (> 126 MB L2)",
                   "wall_ms_per_step": wall_ms / args.steps},
        "e2e": {"value": etoks_all / (ems_max * 1e-3), "unit": "tok/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                "api": "Engine.generate_text(host token lists) -> Request.tokens"},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_source": peak_kind,
                     "traffic": profile_traffic(),
                     "kernel": "varlen paged attention (attn_main_kernel)",
                     "workload": "256 decode seqs ctx log-uniform[256,16384] + 4 prefill chunks "
                                 "of 512 (priors 0/512/1536/3584), 32/8 heads, d128, bf16, "
                                 "16-token blocks, permuted block table, one layer",
                     "algorithmic_bytes": am["bytes"], "ms_per_launch": am["ms_mean"],
                     "prefill_flops": am["prefill_flops"]},
        "secondary": {"upfront10": c2_line},
        "cpu_baseline": cpu,
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
