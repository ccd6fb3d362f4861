"""Host-side pieces of the benchmark module (no GPU)."""
from hayate_b200 import benchmark, workloads


def test_percentile_matches_reference_definition():
    assert benchmark.percentile([], 50) == 0.0
    assert benchmark.percentile([3.0], 95) == 3.0
    assert benchmark.percentile([1.0, 2.0, 3.0, 4.0], 50) == 2.5
    assert abs(benchmark.percentile([1.0, 2.0, 3.0, 4.0], 95) - 3.85) < 1e-12


def test_workloads_are_seeded_and_shaped():
    a, b = workloads.upfront(seed=0), workloads.upfront(seed=0)
    assert [r.prompt for r in a] == [r.prompt for r in b]
    assert len(a) == 10 and all(64 <= len(r.prompt) <= 512 for r in a)
    assert all(r.max_tokens == 256 for r in a)
    p = workloads.poisson(seed=0)
    assert len(p) == 64 and p[0].arrival_s == 0.0
    assert all(x.arrival_s <= y.arrival_s for x, y in zip(p, p[1:]))
    assert all(128 <= len(r.prompt) <= 2048 and 128 <= r.max_tokens <= 512 for r in p)
    m = workloads.attn_micro(seed=0)
    assert len(m.decode_ctx) == 256 and all(256 <= c <= 16384 for c in m.decode_ctx)
    assert m.q_lens()[:4] == [512] * 4 and m.seq_lens_k()[:4] == [512, 1024, 2048, 4096]
    r = workloads.replicas(seed=0, n=16)
    assert all(512 <= len(x.prompt) <= 4096 for x in r)
    reqs = benchmark.make_requests(4, 7, 1337, 160, 320)
    assert len(reqs) == 4 and all(160 <= len(x["prompt"]) <= 320 for x in reqs)


def test_step_trace_charges_only_the_time_a_kernel_extends_the_step():
    """A kernel started early by programmatic dependent launch (the second one
    below starts at 8 while the first runs to 10) is charged from the first's end;
    idle time between kernels is counted as gaps, not charged to either."""
    from hayate_b200.steptrace import critical_path, label
    ev = [("nvjet_tst_128x8_64x12", 0.0, 10.0), ("attn_main_kernel", 8.0, 20.0),
          ("silu_mul_kernel", 25.0, 30.0)]
    excl, dur, cnt, span, gaps = critical_path(ev)
    assert excl[label("nvjet_tst_128x8_64x12")] == 10.0
    assert excl["attention"] == 10.0 and dur["attention"] == 12.0
    assert excl["SiLU*up"] == 5.0
    assert span == 30.0 and gaps == 5.0 and sum(cnt.values()) == 3


def test_splitk_slices_for_decode_sized_bf16_steps_only():
    """o_proj (K 4096) and down_proj (K 9728) split into 8 K slices up to 32 rows
    and 4 up to 128; larger steps, fp32 runs and K that the slices do not divide
    into 8-element multiples keep one GEMM."""
    from types import SimpleNamespace
    import torch
    from hayate_b200.model import Runner
    bf16, fp32 = SimpleNamespace(dtype=torch.bfloat16), SimpleNamespace(dtype=torch.float32)
    assert Runner.splitk_parts(bf16, 16, 4096) == 8
    assert Runner.splitk_parts(bf16, 32, 9728) == 8
    assert Runner.splitk_parts(bf16, 64, 9728) == 4
    assert Runner.splitk_parts(bf16, 129, 4096) == 1
    assert Runner.splitk_parts(fp32, 16, 4096) == 1
    assert Runner.splitk_parts(bf16, 16, 4100) == 1


def test_replica_shares_partition_the_request_set_with_balanced_work():
    """The bench's per-rank workload: the ranks' shares of the world x 256
    replica set (prompts U[512,4096], 256 tokens) are disjoint, cover it
    exactly, and carry near-equal work (prompt + output tokens) under the
    least-outstanding-work rule; at world 1 the share is the whole set."""
    from hayate_b200.workloads import replica_share, replicas
    one = replica_share(1, 0)
    assert len(one) == 256
    assert all(512 <= len(w.prompt) <= 4096 and w.max_tokens == 256 for w in one)
    world = 4
    full = replicas(n=256 * world)
    shares = [replica_share(world, r) for r in range(world)]
    key = lambda w: tuple(w.prompt[:8]) + (len(w.prompt),)   # noqa: E731
    got = sorted(key(w) for s in shares for w in s)
    assert got == sorted(key(w) for w in full)
    work = [sum(len(w.prompt) + w.max_tokens for w in s) for s in shares]
    assert max(work) - min(work) <= 4096 + 256            # within one request's work
