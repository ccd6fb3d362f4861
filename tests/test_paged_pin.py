"""The paged spec (oracle/paged.py) pinned to the reference's own outputs.

The reference has no block pool, packing or slot mapping; ``oracle/paged.py``
specifies them and the CUDA packing kernels are checked against it bit for bit.
These tests tie the spec to the reference through a fixture recorded by running
it (``tests/golden/gen_golden.py --part paged``):

* positions -- every real token the reference feeds through its model carries the
  position id ``arange + cache_len - pad_len`` (qwen.py:66-77); for the token at
  index i of its request's sequence (prompt, then generated tokens) that id is i.
  The spec packs token i of a sequence at position i, so the two agree;
* cache contents -- after a request's last step the reference's compacted cache
  (engine.py:118-141, cache.py:7-10) holds, in column j, the K/V of the token at
  index j.  The spec, driven by this package's scheduler through chunked
  prefill and mixed decode steps, appends each packed token's layer-0 K/V (the
  oracle's per-token projection of its id at its position) at the spec's slot,
  and ``paged.gather`` over the request's block table must give the
  reference's cache back.
"""
import os
from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import GOLDEN
from hayate_b200 import weights as W
from hayate_b200.config import EngineConfig, TINY
from hayate_b200.scheduler import SAMPLE, Scheduler
from oracle import paged as PS
from oracle import reference as R

FIX = np.load(os.path.join(GOLDEN, "tiny_paged_pin.npz"))
SCENARIOS = ("batch5", "long_prompt", "staggered25")
TINY_STD = 0.15


def _requests(name):
    n = int(FIX[f"{name}_nreq"])
    return [(FIX[f"{name}_req{i}_prompt"].tolist(), FIX[f"{name}_req{i}_tokens"].tolist())
            for i in range(n)]


def _reference_positions(name):
    """{request id: {sequence index: position id}} over every real token the
    reference fed through its model; also checks the fed token is the one at
    that index."""
    reqs = _requests(name)
    seen = {i: {} for i in range(len(reqs))}
    for c in range(int(FIX[f"{name}_ncalls"])):
        pos = FIX[f"{name}_call{c}_positions"]
        tok = FIX[f"{name}_call{c}_tokens"]
        ids = FIX[f"{name}_call{c}_ids"]
        pads = FIX[f"{name}_call{c}_pads"]
        cpos = FIX[f"{name}_call{c}_cache_pos"]
        T = pos.shape[1]
        for b, rid in enumerate(ids.tolist()):
            prompt, gen = reqs[rid]
            seq = prompt + gen
            for col in range(int(pads[b]), T):
                idx = int(cpos[b]) + col - int(pads[b])
                assert int(tok[b, col]) == seq[idx]
                seen[rid][idx] = int(pos[b, col])
    return seen


@pytest.mark.parametrize("name", SCENARIOS)
def test_reference_position_of_token_i_is_i(name):
    seen = _reference_positions(name)
    for rid, (prompt, gen) in enumerate(_requests(name)):
        fed = len(prompt) + len(gen) - 1          # the last sampled token is never fed
        assert sorted(seen[rid]) == list(range(fed))
        assert all(p == i for i, p in seen[rid].items())


@pytest.fixture(scope="module")
def layer0():
    hw = W.sequential_seeded(TINY, 0, std=TINY_STD)
    Wt = R.RefWeights.from_host(hw, torch.float32)
    return Wt


def _layer0_kv(Wt, ids, positions):
    """Layer-0 K (after k_norm and RoPE) and V of each token, from its id and
    position alone (attention.py:36-48 for one token; block.py:23)."""
    p = Wt.layers[0]
    x = F.embedding(torch.as_tensor(ids, dtype=torch.long), Wt.embed)[None]
    h = R.rms_norm(x, p["input_layernorm"], Wt.eps)
    T = len(ids)
    k = F.linear(h, p["k_proj"]).view(1, T, Wt.num_kv_heads, Wt.head_dim)
    v = F.linear(h, p["v_proj"]).view(1, T, Wt.num_kv_heads, Wt.head_dim)
    k = R.rms_norm(k, p["k_norm"], Wt.eps).transpose(1, 2)
    k = R.rope(k, Wt.cos, Wt.sin, torch.as_tensor(positions, dtype=torch.long)[None])
    return k[0].transpose(0, 1).numpy(), v[0].numpy()     # (T, Hkv, D)


@pytest.mark.parametrize("name", SCENARIOS)
def test_spec_positions_and_cache_match_reference(name, layer0):
    """The spec, driven by the engine's scheduler (16-token prefill chunks, at
    most 6 live requests, a 40-token step budget, block reuse after frees),
    packs each token at the reference's position for it and rebuilds each
    request's compacted cache from its blocks."""
    ref_pos = _reference_positions(name)
    reqs = _requests(name)
    Hkv, D = TINY.num_kv_heads, TINY.head_dim
    cfg = EngineConfig(max_num_seqs=6, max_batched_tokens=40, prefill_chunk=16,
                       max_model_len=1024)
    max_reqs, num_blocks = cfg.max_num_seqs + 1, 160
    sch = Scheduler(cfg, num_blocks, max_reqs)
    st = PS.PagedState(max_reqs, cfg.max_model_len + 1, cfg.max_model_len // 16, num_blocks)
    cache = np.zeros((num_blocks, 2, Hkv, 16, D), np.float32)
    live = []
    for i, (prompt, gen) in enumerate(reqs):
        r = SimpleNamespace(id=i, prompt_tokens=prompt, max_tokens=len(gen), slot=-1, _blocks=0,
                            cache_pos=0, is_prefill=True, is_completed=False,
                            _last_launched=False, tokens=[])
        sch.check_request(r)
        sch.waiting.append(r)
    checked, steps = 0, 0
    while sch.waiting or sch.running:
        for r in sch.admit():
            st.req_tokens[r.slot, :] = 0
            st.req_tokens[r.slot, :len(r.prompt_tokens)] = r.prompt_tokens
            live.append(r)
        plan = sch.schedule()
        assert plan.num_seqs > 0
        sched = PS.make_sched([e.req.slot for e in plan.entries], [e.start for e in plan.entries],
                              [e.q_len for e in plan.entries], [e.flags for e in plan.entries])
        T = plan.num_tokens
        out = PS.pack(st, sched, T)
        by_slot = {e.req.slot: e.req for e in plan.entries}
        rows = np.repeat(np.arange(plan.num_seqs), [e.q_len for e in plan.entries])
        for k in range(T):
            r = plan.entries[rows[k]].req
            p = int(out["positions"][k])
            assert ref_pos[r.id][p] == p                         # qwen.py:66-77
            assert int(out["input_ids"][k]) == (r.prompt_tokens + reqs[r.id][1])[p]
        kk, vv = _layer0_kv(layer0, out["input_ids"], out["positions"])
        PS.kv_append(cache, kk, vv, out["slot_mapping"])
        # "sample": the reference's next token for every sequence that samples
        nxt = np.array([reqs[plan.entries[i].req.id][1][len(plan.entries[i].req.tokens)]
                        for i in out["sample_seq"]], np.int32)
        PS.commit(st, nxt, out["sample_seq"], sched)
        done = []
        for e in plan.entries:
            r = e.req
            r.cache_pos = e.start + e.q_len
            if e.flags & SAMPLE:
                r.is_prefill = False
                r.tokens.append(reqs[r.id][1][len(r.tokens)])
                if len(r.tokens) >= sch.token_limit(r):
                    r.is_completed = r._last_launched = True
                    done.append(r)
        for r in done:
            n = len(r.prompt_tokens) + len(r.tokens) - 1
            k_got, v_got = PS.gather(cache, st.block_tables[r.slot], n)   # (Hkv, n, D)
            k_ref = FIX[f"{name}_req{r.id}_k"]                           # (Hkv, n, 4)
            v_ref = FIX[f"{name}_req{r.id}_v"]
            assert k_ref.shape == (Hkv, n, k_ref.shape[2])
            np.testing.assert_allclose(k_got[..., :k_ref.shape[2]], k_ref, rtol=1e-5, atol=1e-5)
            np.testing.assert_allclose(v_got[..., :v_ref.shape[2]], v_ref, rtol=1e-5, atol=1e-5)
            PS.free(st, [r.slot])
            sch.release(r)
            checked += 1
        steps += 1
        assert steps < 2000
    assert checked == len(reqs)
    assert st.free_top == num_blocks                   # every block came back
