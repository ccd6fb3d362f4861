"""The CPU oracle against fixtures produced by running the reference itself."""
import json
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from hayate_b200.config import TINY, QWEN3_4B
from hayate_b200 import weights as W
from oracle import reference as R

TINY_STD = json.load(open(os.path.join(GOLDEN, "tiny_engine.json")))["std"]


@pytest.fixture(scope="module")
def tiny_weights():
    return W.sequential_seeded(TINY, 0, std=TINY_STD)


def test_rope_tables_match_reference():
    f = np.load(os.path.join(GOLDEN, "qk_norm_rope.npz"))
    cos, sin = R.rope_tables(128, QWEN3_4B.rope_theta, QWEN3_4B.max_position_embeddings)
    pos = torch.from_numpy(f["positions"])
    assert torch.equal(cos[pos], torch.from_numpy(f["cos_rows"]))
    assert torch.equal(sin[pos], torch.from_numpy(f["sin_rows"]))
    # the second half duplicates the first (rope.py:10), so kernels keep 64 columns
    assert torch.equal(cos[:, :64], cos[:, 64:])


@pytest.mark.parametrize("tag,dt", [("bf16", torch.bfloat16), ("fp32", torch.float32)])
def test_qk_norm_rope_matches_reference(tag, dt):
    f = np.load(os.path.join(GOLDEN, "qk_norm_rope.npz"))

    def t(name):
        a = torch.from_numpy(f[f"{tag}_{name}"])
        return a.view(torch.bfloat16) if dt == torch.bfloat16 else a
    cos, sin = R.rope_tables(128, QWEN3_4B.rope_theta, QWEN3_4B.max_position_embeddings)
    qo, ko = R.qk_norm_rope(t("q"), t("k"), t("wq"), t("wk"), cos, sin,
                            torch.from_numpy(f["positions"]), QWEN3_4B.rms_norm_eps)
    assert torch.equal(qo, t("q_out"))
    assert torch.equal(ko, t("k_out"))


def test_forward_matches_reference(tiny_weights):
    f = np.load(os.path.join(GOLDEN, "tiny_forward.npz"))
    Wt = R.RefWeights.from_host(tiny_weights, torch.float32)
    # call 0: left-padded prefill
    logits, nk, nv = R.forward(Wt, torch.from_numpy(f["c0_token_ids"]),
                               pad_lengths=torch.from_numpy(f["c0_pad_lengths"]))
    assert torch.equal(logits, torch.from_numpy(f["c0_logits"]))
    assert torch.equal(nk, torch.from_numpy(f["c0_new_k"]))
    assert torch.equal(nv, torch.from_numpy(f["c0_new_v"]))
    # call 1: decode over the padded, stacked caches
    logits, nk, nv = R.forward(Wt, torch.from_numpy(f["c1_token_ids"]),
                               torch.from_numpy(f["c1_prev_k"]), torch.from_numpy(f["c1_prev_v"]),
                               torch.from_numpy(f["c1_cache_lens"]))
    assert torch.equal(logits, torch.from_numpy(f["c1_logits"]))
    assert torch.equal(nv, torch.from_numpy(f["c1_new_v"]))


def _run_ref_scenario(Wt, sc):
    eng = R.RefEngine(Wt, record_margins=True)
    if sc["kind"] == "upfront":
        reqs = eng.run([r["prompt"] for r in sc["requests"]], sc["requests"][0]["max_tokens"])
        return reqs
    arrivals = sorted(((r["arrival_step"], i, r) for i, r in enumerate(sc["requests"])))
    out = [None] * len(sc["requests"])
    step = 0
    while arrivals or eng.current_batch or eng.pool:
        while arrivals and arrivals[0][0] <= step:
            _, i, r = arrivals.pop(0)
            out[i] = eng.add(r["prompt"], r["max_tokens"])
        eng.step()
        step += 1
    return out


@pytest.mark.parametrize("name", ["single", "batch5", "max_tokens_one", "staggered25"])
def test_engine_loop_matches_reference(tiny_weights, name):
    g = json.load(open(os.path.join(GOLDEN, "tiny_engine.json")))
    sc = g["scenarios"][name]
    reqs = _run_ref_scenario(R.RefWeights.from_host(tiny_weights, torch.float32), sc)
    for r, want in zip(reqs, sc["requests"]):
        assert r.tokens == want["tokens"]
        np.testing.assert_allclose(r.margins, want["margins"], rtol=0, atol=0)
