"""The reference's benchmark modes run end to end on the engine (small sizes)."""
import pytest

from hayate_b200 import benchmark

pytestmark = pytest.mark.gpu


def test_benchmark_modes_small():
    rows = benchmark.main(["3", "--repetitions", "1", "--max-tokens", "8",
                           "--min-prompt-tokens", "16", "--max-prompt-tokens", "40",
                           "--arrival-gap-ms", "5", "--modes", "single,upfront,staggered"])
    names = [t for t, _ in rows]
    assert names == ["single request", "submit all upfront", "staggered arrivals"]
    for _, r in rows:
        assert r["generated_tokens"] > 0 and r["elapsed"] > 0
        assert len(r["latencies"]) >= 1
    # single mode: 3 requests x 8 tokens; upfront: one run of 3 x 8
    assert rows[0][1]["generated_tokens"] == 24
    assert rows[1][1]["generated_tokens"] == 24


@pytest.mark.parametrize("op", ["qk_norm_rope", "kv_append", "pack", "argmax", "attention",
                                "add_rms_norm", "silu_mul"])
def test_operator_microbench_small(op):
    from hayate_b200.microbench import run_op
    r = run_op(op, iters=2, n_decode=16, prefill=True, tokens=16 + 512)
    assert r["op"] == op and r["ms_mean"] > 0 and r["bytes"] > 0


@pytest.mark.parametrize("op", ["qk_norm_rope", "kv_append", "argmax", "add_rms_norm",
                                "silu_mul"])
def test_row_kernel_microbench_streamed(op):
    """The streamed timing mode: launches on input copies larger than L2,
    replayed from one CUDA graph (prefill-sized cases, so the streamed
    add+RMSNorm and QK-norm+RoPE kernels run)."""
    from hayate_b200.microbench import run_op
    r = run_op(op, iters=2, n_decode=16, prefill=True, tokens=16 + 2048, stream=True)
    assert r["op"] == op and r["ms_mean"] > 0 and r["bytes"] > 0 and r["stream"]
