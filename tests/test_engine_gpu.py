"""The engine end to end on a B200 against the reference's greedy tokens."""
import json
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from hayate_b200 import weights as W
from hayate_b200.config import EngineConfig, QWEN3_4B, TINY
from hayate_b200.engine import Engine, Request

pytestmark = pytest.mark.gpu

TINY_GOLD = json.load(open(os.path.join(GOLDEN, "tiny_engine.json")))


def tiny_engine(dtype, graphs, chunk=64, max_seqs=32, tokenizer=None, max_model_len=1024,
                engine_cls=Engine):
    ecfg = EngineConfig(max_num_seqs=max_seqs, max_batched_tokens=256, prefill_chunk=chunk,
                        num_kv_blocks=512, max_model_len=max_model_len, cuda_graphs=graphs)
    hw = W.exact_seeded(TINY, 0, std=TINY_GOLD["std"])
    return engine_cls("tiny", model_config=TINY, engine_config=ecfg, dtype=dtype, weights=hw,
                      tokenizer=tokenizer)


class IdTokenizer:
    """Token-id prompts; ``eos_token_id`` as the reference's tokenizer has one."""
    pad_token_id = 0

    def __init__(self, eos_token_id=None):
        self.eos_token_id = eos_token_id

    def encode(self, prompt):
        return list(prompt)

    def decode(self, ids, skip_special_tokens=True):
        return " ".join(map(str, ids))


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


EOS_GOLD = json.load(open(os.path.join(GOLDEN, "tiny_eos.json")))


@pytest.mark.parametrize("graphs", [False, True])
@pytest.mark.parametrize("name", sorted(EOS_GOLD["scenarios"]))
def test_tiny_fp32_stops_at_eos_like_reference(name, graphs):
    """With the tokenizer's eos id set, a request completes on the step that
    samples eos (engine.py:76-77): the same tokens as the reference, eos last,
    nothing after it, and its slot freed for the requests behind it."""
    sc = EOS_GOLD["scenarios"][name]
    eos = sc["eos_token_id"]
    eng = tiny_engine(torch.float32, graphs, tokenizer=IdTokenizer(eos))
    reqs = run_scenario(eng, sc)
    early = 0
    for r, want in zip(reqs, sc["requests"]):
        assert r.is_completed and r.tokens == want["tokens"], (r.id, r.tokens, want["tokens"])
        if len(r.tokens) < want["max_tokens"]:
            assert r.tokens[-1] == eos and eos not in r.tokens[:-1]
            assert r.response is not None
            early += 1
    assert early > 0
    assert not eng.scheduler.running and eng.check_device_errors() == 0


def test_output_capped_at_max_model_len():
    """max_tokens past max_model_len: the request ends at the length limit with
    no device error (its token row and block table hold exactly that much)."""
    eng = tiny_engine(torch.bfloat16, True, max_model_len=64)
    r = eng.generate_text(list(range(1, 41)), max_tokens=100)
    assert r.is_completed and len(r.tokens) == 24
    rs = eng.generate_text([list(range(1, 60)), [7] * 10], max_tokens=30)
    assert [len(x.tokens) for x in rs] == [5, 30]
    assert eng.check_device_errors() == 0


class LogitsEngine(Engine):
    """Overrides ``sample`` as the reference's hook (engine.py:69-71): receives
    each step's last-token logits and picks greedily with torch."""

    def __init__(self, *a, **kw):
        super().__init__(*a, **kw)
        self.seen = []

    def sample(self, logits):
        self.seen.append(logits.detach().clone())
        return torch.argmax(logits, dim=-1, keepdim=True)


def test_model_boundary_returns_the_reference_last_token_logits():
    """The model half of a step returns the logits of each sampled sequence's
    last token: equal (fp32) to the reference model's ``logits[:, -1, :]`` for
    its first prefill call and its first decode call (qwen.py:46-59,
    engine.py:143-163), and the tokens a custom ``sample`` picks are committed."""
    f = np.load(os.path.join(GOLDEN, "tiny_forward.npz"))
    lens = f["prompt_lens"].tolist()
    flat = f["prompts_flat"].tolist()
    prompts, o = [], 0
    for n in lens:
        prompts.append(flat[o:o + n])
        o += n
    eng = tiny_engine(torch.float32, True, engine_cls=LogitsEngine)
    assert not eng.use_graphs                    # a custom sampler is not captured
    reqs = eng.generate_text(prompts, max_tokens=3)
    assert len(eng.seen) == 3                   # prefill, then two decode steps
    for step, key in ((0, "c0_logits"), (1, "c1_logits")):
        want = torch.from_numpy(f[key][:, -1, :])
        got = eng.seen[step].float().cpu()
        assert got.shape == want.shape
        torch.testing.assert_close(got, want, rtol=1e-4, atol=1e-4)
    plain = tiny_engine(torch.float32, True).generate_text(prompts, max_tokens=3)
    assert [r.tokens for r in reqs] == [r.tokens for r in plain]
    assert eng.check_device_errors() == 0


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


def test_decode_graphs_of_more_than_128_rows_give_the_eager_tokens():
    """150 sequences decoding at once: the bucket-160 decode graph samples 160
    rows, so its LM head + argmax runs on CTA pairs (clusters of two) inside the
    graph; its tokens must equal those of the same engine without graphs."""
    g = torch.Generator().manual_seed(11)
    prompts = [torch.randint(1, TINY.vocab_size, (8,), generator=g).tolist() for _ in range(150)]
    toks = []
    for graphs in (True, False):
        eng = tiny_engine(torch.bfloat16, graphs, max_seqs=160)
        # 256 tokens a step: all 150 prompts are in by the 7th step, before the
        # first request's 16 tokens are done, so later steps decode 150 rows
        reqs = eng.generate_text(prompts, max_tokens=16)
        assert all(r.is_completed and len(r.tokens) == 16 for r in reqs)
        assert eng.check_device_errors() == 0
        if graphs:
            assert 160 in eng._graphs
        toks.append([r.tokens for r in reqs])
    assert toks[0] == toks[1]


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


def _tokens_match(reqs, want, ntok):
    for r, w in zip(reqs, want):
        got, exp = r.tokens[:ntok], w["tokens"][:ntok]
        if got != exp:
            i = next(j for j in range(ntok) if got[j] != exp[j])
            pytest.fail(f"request {r.id}: first divergence at token {i} "
                        f"(reference top-2 margin there {w['margins'][i]:.3g})")


@pytest.mark.parametrize("case,ntok", [("single", 32), ("upfront", 32)])
def test_qwen3_4b_fp32_greedy_matches_reference(full_fp32_engine, case, ntok):
    eng = full_fp32_engine
    want = FULL["cases"][case]
    reqs = eng.generate_text([r["prompt"] for r in want], max_tokens=ntok)
    reqs = reqs if isinstance(reqs, list) else [reqs]
    _tokens_match(reqs, want, ntok)
    assert eng.check_device_errors() == 0


CHUNKED = json.load(open(os.path.join(GOLDEN, "full_chunked.json")))


def test_qwen3_4b_fp32_chunked_prefill_matches_reference(full_fp32_engine):
    """The first 6 requests of the Poisson workload (prompts of 1330, 1861,
    1125, 345, 280 and 256 tokens): the engine splits the three long prompts
    into 512-token chunks, runs them in steps beside the short requests'
    decodes, and must give the reference's fp32 greedy tokens (its one padded
    prefill of all 6, then decodes) for the first 32 tokens of each."""
    eng = full_fp32_engine
    want = CHUNKED["requests"]
    chunk = eng.ecfg.prefill_chunk
    assert sum(len(w["prompt"]) > chunk for w in want) >= 3
    steps0, tok0 = eng.steps, eng.prompt_tokens_computed
    reqs = eng.generate_text([w["prompt"] for w in want], max_tokens=32)
    assert eng.prompt_tokens_computed - tok0 == sum(len(w["prompt"]) for w in want)
    assert eng.steps - steps0 > 32              # chunked prefill took extra mixed steps
    _tokens_match(reqs, want, 32)
    assert eng.check_device_errors() == 0
