"""The engine end to end on a B200 against the reference's greedy tokens."""
import json
import os

import pytest
import torch

from conftest import GOLDEN
from hayate_b200 import weights as W
from hayate_b200.config import EngineConfig, QWEN3_4B, TINY
from hayate_b200.engine import Engine, Request

pytestmark = pytest.mark.gpu

TINY_GOLD = json.load(open(os.path.join(GOLDEN, "tiny_engine.json")))


def tiny_engine(dtype, graphs, chunk=64, max_seqs=32):
    ecfg = EngineConfig(max_num_seqs=max_seqs, max_batched_tokens=256, prefill_chunk=chunk,
                        num_kv_blocks=512, max_model_len=1024, cuda_graphs=graphs)
    hw = W.exact_seeded(TINY, 0, std=TINY_GOLD["std"])
    return Engine("tiny", model_config=TINY, engine_config=ecfg, dtype=dtype, weights=hw)


def run_scenario(eng, sc):
    if sc["kind"] == "upfront":
        reqs = eng.generate_text([r["prompt"] for r in sc["requests"]],
                                 max_tokens=sc["requests"][0]["max_tokens"])
        return reqs if isinstance(reqs, list) else [reqs]
    arrivals = sorted((r["arrival_step"], i) for i, r in enumerate(sc["requests"]))
    out = [None] * len(sc["requests"])
    step = 0
    while arrivals or eng.current_batch or not eng.pool.empty():
        while arrivals and arrivals[0][0] <= step:
            _, i = arrivals.pop(0)
            r = sc["requests"][i]
            out[i] = Request(id=eng.request_id, prompt=r["prompt"], max_tokens=r["max_tokens"])
            eng.request_id += 1
            eng.add_request(out[i])
        eng.generate()
        step += 1
    return out


@pytest.mark.parametrize("graphs", [False, True])
@pytest.mark.parametrize("name", sorted(TINY_GOLD["scenarios"]))
def test_tiny_fp32_tokens_equal_reference(name, graphs):
    eng = tiny_engine(torch.float32, graphs)
    sc = TINY_GOLD["scenarios"][name]
    reqs = run_scenario(eng, sc)
    for r, want in zip(reqs, sc["requests"]):
        assert r.is_completed
        assert r.tokens == want["tokens"], (r.id, len(r.prompt_tokens))
    assert eng.check_device_errors() == 0
    if graphs and name in ("batch5", "staggered25"):
        assert eng.graph_steps > 0


def test_tiny_bf16_first_tokens_where_margin_is_clear():
    eng = tiny_engine(torch.bfloat16, True)
    checked = 0
    for sc in TINY_GOLD["scenarios"].values():
        reqs = run_scenario(eng, sc)
        for r, want in zip(reqs, sc["requests"]):
            assert r.is_completed and len(r.tokens) == len(want["tokens"])
            if want["margins"][0] > 0.15:
                assert r.tokens[0] == want["tokens"][0]
                checked += 1
    assert checked >= 10
    assert eng.check_device_errors() == 0


def test_engine_api_shapes():
    eng = tiny_engine(torch.bfloat16, False)
    one = eng.generate_text([5, 6, 7], max_tokens=3)
    assert isinstance(one, Request) and len(one.tokens) == 3 and one.is_completed
    many = eng.generate_text([[1, 2], [3]], max_tokens=2)
    assert isinstance(many, list) and all(len(r.tokens) == 2 for r in many)
    assert eng.generate() is False
    s = eng.generate_text("hi", max_tokens=1)
    assert s.prompt_tokens == list(b"hi") and s.response is not None


def test_trace_ranges_leave_tokens_unchanged():
    """NVTX ranges around the step phases change nothing the engine computes."""
    sc = TINY_GOLD["scenarios"][sorted(TINY_GOLD["scenarios"])[0]]
    plain = run_scenario(tiny_engine(torch.float32, True), sc)
    eng = tiny_engine(torch.float32, True)
    eng.trace = True
    traced = run_scenario(eng, sc)
    assert [r.tokens for r in traced] == [r.tokens for r in plain]


def test_graphs_captured_ahead_give_the_same_tokens():
    """Decode graphs captured up front (padding-slot schedules) replay real steps."""
    name = sorted(TINY_GOLD["scenarios"])[-1]
    sc = TINY_GOLD["scenarios"][name]
    eng = tiny_engine(torch.float32, True)
    assert eng.capture_graphs() == len(eng._graphs) > 0
    got = run_scenario(eng, sc)
    want = [r["tokens"] for r in sc["requests"]]
    assert [r.tokens for r in got] == want
    assert eng.check_device_errors() == 0


_PDL_SCRIPT = """
import json, sys, torch
sys.path.insert(0, {tests!r})
from test_engine_gpu import tiny_engine, run_scenario, TINY_GOLD
sc = TINY_GOLD["scenarios"][{name!r}]
eng = tiny_engine(torch.bfloat16, True)
print(json.dumps([r.tokens for r in run_scenario(eng, sc)]))
"""


def test_programmatic_launch_changes_no_token():
    """The step's kernels start early under programmatic dependent launch and wait
    for their inputs on the device; the same bf16 run without it (HY_PDL=0, read
    once per process) gives the same tokens."""
    import subprocess
    import sys
    name = sorted(TINY_GOLD["scenarios"])[-1]
    here = os.path.dirname(os.path.abspath(__file__))
    with_pdl = [r.tokens for r in run_scenario(tiny_engine(torch.bfloat16, True),
                                               TINY_GOLD["scenarios"][name])]
    env = dict(os.environ, HY_PDL="0")
    out = subprocess.run([sys.executable, "-c", _PDL_SCRIPT.format(tests=here, name=name)],
                         env=env, capture_output=True, text=True, timeout=600,
                         cwd=os.path.dirname(here))
    assert out.returncode == 0, out.stderr[-2000:]
    without = json.loads(out.stdout.strip().splitlines()[-1])
    assert with_pdl == without


def _tiny_cached(prefix_caching, num_kv_blocks=512, max_model_len=1024):
    ecfg = EngineConfig(max_num_seqs=8, max_batched_tokens=256, prefill_chunk=64,
                        num_kv_blocks=num_kv_blocks, max_model_len=max_model_len,
                        cuda_graphs=True, prefix_caching=prefix_caching)
    hw = W.exact_seeded(TINY, 0, std=TINY_GOLD["std"])
    return Engine("tiny", model_config=TINY, engine_config=ecfg, dtype=torch.float32, weights=hw)


def test_prefix_caching_shares_blocks_and_keeps_tokens():
    """Prompts sharing a 100-token prefix: once the first has run, the others take
    its 6 full blocks from the cache, compute 96 prompt tokens fewer each, and
    produce the tokens of an engine without the cache."""
    import random
    rng = random.Random(7)
    prefix = [rng.randrange(TINY.vocab_size) for _ in range(100)]
    prompts = [prefix + [rng.randrange(TINY.vocab_size) for _ in range(rng.randint(1, 30))]
               for _ in range(6)]
    runs = {}
    for on in (False, True):
        eng = _tiny_cached(on)
        first = eng.generate_text(prompts[0], max_tokens=8)
        rest = eng.generate_text(prompts[1:], max_tokens=8)
        assert eng.check_device_errors() == 0
        runs[on] = ([first.tokens] + [r.tokens for r in rest], eng.prompt_tokens_computed, eng)
    assert runs[True][0] == runs[False][0]
    assert runs[False][1] - runs[True][1] == 5 * 96
    assert runs[True][2].prefix_cache.held >= 6


def test_prefix_caching_evicts_when_the_pool_is_short():
    """Waves of distinct prompts fill a small pool with cached blocks; admissions
    evict the idle ones and the tokens stay those of an engine without the cache."""
    import random
    rng = random.Random(11)
    waves = [[[rng.randrange(TINY.vocab_size) for _ in range(rng.randint(60, 120))]
              for _ in range(3)] for _ in range(5)]
    out = {}
    for on in (False, True):
        eng = _tiny_cached(on, num_kv_blocks=40, max_model_len=200)
        toks = []
        for w in waves:
            toks += [r.tokens for r in eng.generate_text(w, max_tokens=6)]
        assert eng.check_device_errors() == 0
        out[on] = toks
        if on:
            assert eng.prefix_cache.held <= 39
    assert out[True] == out[False]


FULL = json.load(open(os.path.join(GOLDEN, "full_greedy.json")))


@pytest.fixture(scope="module")
def full_fp32_engine():
    hw = W.exact_seeded(QWEN3_4B, 0)
    fp = W.fingerprint(hw)
    for k, v in FULL["fingerprint"].items():
        assert fp[k] == v, f"weights differ from the fixture's at {k}"
    ecfg = EngineConfig(max_num_seqs=16, max_batched_tokens=4096, prefill_chunk=512,
                        num_kv_blocks=2048, max_model_len=2048, cuda_graphs=True)
    eng = Engine("Qwen/Qwen3-4B", engine_config=ecfg, dtype=torch.float32, weights=hw)
    del hw
    yield eng
    del eng
    torch.cuda.empty_cache()


@pytest.mark.parametrize("case,ntok", [("single", 32), ("upfront", 32)])
def test_qwen3_4b_fp32_greedy_matches_reference(full_fp32_engine, case, ntok):
    eng = full_fp32_engine
    want = FULL["cases"][case]
    reqs = eng.generate_text([r["prompt"] for r in want], max_tokens=ntok)
    reqs = reqs if isinstance(reqs, list) else [reqs]
    for r, w in zip(reqs, want):
        got, exp = r.tokens[:ntok], w["tokens"][:ntok]
        if got != exp:
            i = next(j for j in range(ntok) if got[j] != exp[j])
            pytest.fail(f"request {r.id}: first divergence at token {i} "
                        f"(reference top-2 margin there {w['margins'][i]:.3g})")
    assert eng.check_device_errors() == 0
