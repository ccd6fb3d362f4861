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
