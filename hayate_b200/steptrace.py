"""Critical path of the engine's steps, per kernel.

``python -m hayate_b200.steptrace [--steps 10]`` runs the upfront workload's 10
requests (bf16 Qwen3-4B, random weights) into their decode phase, records
``--steps`` decode steps with the torch profiler (CUPTI kernel timestamps, no
ncu) and charges each kernel only for the time it extends the step: its end
minus the later of its own start and the previous kernel's end.  Kernels that
programmatic dependent launch starts early (before the previous kernel ends)
are therefore not charged for the overlap, which plain per-kernel durations are.

``python -m hayate_b200.steptrace --replica-share`` does the same over one
complete run of a replica's share of the 2048-request workload (256 requests,
prompts U[512,4096], 256 tokens each; one warm-up run first).
"""
from __future__ import annotations

import argparse
import collections

import torch

# kernel-name fragments -> row label, first match wins
LABELS = (
    ("attn_main", "attention"),
    ("add_rms_norm_kernel<__nv_bfloat16, true", "add+RMSNorm, split-K partials"),
    ("add_rms_norm", "add+RMSNorm"),
    ("qk_norm_rope", "QK-norm+RoPE (+KV append)"),
    ("silu_mul", "SiLU*up"),
    ("nvjet_tss_192x16", "cuBLAS o/down (batched over K slices)"),
    ("nvjet_tst_192x16", "cuBLAS gate/up"),
    ("nvjet_tst_128x8", "cuBLAS qkv"),
    ("nvjet_tst_384x16", "cuBLAS LM head"),
    ("nvjet", "cuBLAS (other shapes)"),
    ("gemm", "cuBLAS (other shapes)"),
    ("indexSelect", "embedding / row gather"),
    ("plan_kernel", "attention plan"),
    ("pack_kernel", "pack"),
    ("lm_head_argmax", "LM head + argmax (fused)"),
    ("argmax", "argmax"),
    ("commit", "commit"),
    ("Memcpy", "memcpy"),
)


def label(name: str) -> str:
    for frag, lab in LABELS:
        if frag in name:
            return lab
    return name[:48]


def critical_path(events):
    """events: (name, start_us, end_us) sorted by start -> (per-label exclusive
    time, duration, count), total span, gaps between kernels."""
    excl = collections.defaultdict(float)
    dur = collections.defaultdict(float)
    cnt = collections.Counter()
    prev_end, gaps = None, 0.0
    for name, s, t in events:
        lab = label(name)
        base = s if prev_end is None else max(prev_end, s)
        if prev_end is not None and s > prev_end:
            gaps += s - prev_end
        excl[lab] += max(0.0, t - base)
        dur[lab] += t - s
        cnt[lab] += 1
        prev_end = t if prev_end is None else max(prev_end, t)
    span = events[-1][2] - events[0][1] if events else 0.0
    return excl, dur, cnt, span, gaps


def report(ev, title, per):
    excl, dur, cnt, span, gaps = critical_path(ev)
    print(f"{title}: {span / per:.1f} us per {'step' if per > 1 else 'run'}, gaps between "
          f"kernels {gaps / per:.1f} us")
    for lab, x in sorted(excl.items(), key=lambda kv: -kv[1]):
        print(f"{lab:40s} {cnt[lab] / per:8.1f}/{'step' if per > 1 else 'run'}  "
              f"{x / cnt[lab]:8.2f} us excl ({100 * x / span:4.1f}%)  "
              f"{dur[lab] / cnt[lab]:8.2f} us duration")


def attention_by_step(events, log, cfg):
    """Attention launches grouped by engine step (in launch order; a step whose
    sequences sample nothing skips the last layer's): time and the KV bytes of
    decode-only steps (every key of every sequence read once per layer)."""
    att = [(s, t) for n, s, t in events if "attn_main" in n]
    L = cfg.num_layers
    kv_token_layer = 2 * cfg.num_kv_heads * cfg.head_dim * 2        # K and V, bf16
    k = 0
    dec_us = dec_bytes = mix_us = 0.0
    n_dec = n_mix = 0
    for S, T, ns, decode_only, keys in log:
        n = L if ns > 0 else L - 1
        us = sum(t - s for s, t in att[k:k + n])
        k += n
        if decode_only:
            dec_us += us
            dec_bytes += keys * kv_token_layer * n
            n_dec += 1
        else:
            mix_us += us
            n_mix += 1
    if k != len(att):
        print(f"(attention launches {len(att)} != {k} expected from the step log)")
    if n_dec:
        print(f"decode-only steps: {n_dec}, attention {dec_us / 1e3:.1f} ms for "
              f"{dec_bytes / 1e9:.1f} GB of K/V = {dec_bytes / (dec_us * 1e-6) / 1e9:.0f} GB/s")
    if n_mix:
        print(f"steps with prefill chunks: {n_mix}, attention {mix_us / 1e3:.1f} ms")


def _cuda_events(prof):
    return sorted(((e.name, e.time_range.start, e.time_range.end) for e in prof.events()
                   if e.device_type == torch.autograd.DeviceType.CUDA), key=lambda x: x[1])


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--replica-share", action="store_true",
                    help="profile one full run of a replica's 256-request share")
    args = ap.parse_args()
    from torch.profiler import ProfilerActivity, profile

    from .config import EngineConfig
    from .engine import Engine, Request
    from .workloads import upfront
    if args.replica_share:
        from .benchmark import replica_engine_config
        from .workloads import replica_share
        share = replica_share(1, 0)
        eng = Engine("Qwen/Qwen3-4B", engine_config=replica_engine_config(share),
                     weights="device")
        eng.capture_graphs()
        prompts = [torch.tensor(w.prompt, dtype=torch.int32, device=eng.device) for w in share]
        eng.generate_text(prompts, max_tokens=256)          # warm-up run
        torch.cuda.synchronize()
        s0 = eng.steps
        eng.step_log = []
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            eng.generate_text(prompts, max_tokens=256)
            torch.cuda.synchronize()
        ev = _cuda_events(prof)
        report(ev, f"one run of {len(share)} requests, {eng.steps - s0} engine "
               f"steps ({eng.graph_steps} graph-replayed in all runs)", 1)
        attention_by_step(ev, eng.step_log, eng.cfg)
        return
    ecfg = EngineConfig(max_num_seqs=16, max_batched_tokens=8192, prefill_chunk=512,
                        num_kv_blocks=1024, max_model_len=1024, cuda_graphs=True,
                        ignore_eos=True)
    eng = Engine("Qwen/Qwen3-4B", engine_config=ecfg, weights="device")
    prompts = [r.prompt for r in upfront(seed=0)]
    eng.generate_text(prompts, max_tokens=64)            # warm-up: graphs captured
    for p in prompts:
        eng.add_request(Request(id=eng.request_id, prompt=p, max_tokens=args.steps + 50))
        eng.request_id += 1
    eng.generate()                                      # prefill
    eng.generate()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(args.steps):
            eng.generate()
        torch.cuda.synchronize()
    report(_cuda_events(prof), f"{args.steps} decode steps of 10 sequences", args.steps)


if __name__ == "__main__":
    main()
