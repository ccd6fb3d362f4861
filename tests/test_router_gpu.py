"""The router's GPU path: engine replicas in their own processes (spawned,
one per GPU) behind ``hayate_b200.router.Router``, as the replicas benchmark
mode and the multi-GPU configuration run them.  The tiny fp32 model's
replicas must return the reference's greedy tokens for every request,
whichever replica served it.
"""
import json
import os
import time

import pytest
import torch

from conftest import GOLDEN
from hayate_b200 import weights as W
from hayate_b200.config import EngineConfig, TINY
from hayate_b200.router import Router

pytestmark = pytest.mark.gpu

TINY_GOLD = json.load(open(os.path.join(GOLDEN, "tiny_engine.json")))


def test_router_replicas_return_the_reference_tokens():
    n = min(2, torch.cuda.device_count())
    ecfg = EngineConfig(max_num_seqs=32, max_batched_tokens=256, prefill_chunk=64,
                        num_kv_blocks=512, max_model_len=1024, cuda_graphs=True)
    kwargs = dict(model_name="tiny", model_config=TINY, engine_config=ecfg,
                  dtype=torch.float32, weights=W.exact_seeded(TINY, 0, std=TINY_GOLD["std"]))
    reqs = [r for name in ("batch5", "long_prompt", "max_tokens_one")
            for r in TINY_GOLD["scenarios"][name]["requests"]]
    with Router(n, factory_kwargs=kwargs) as router:
        deadline = time.time() + 600
        while not all(router.ready):
            assert all(router.alive), "a replica process exited before it was ready"
            assert time.time() < deadline, "replicas not ready"
            router.poll(0.5)
        ids = [router.submit(r["prompt"], r["max_tokens"]) for r in reqs]
        res = router.wait_all(timeout=600)
        assert not router.failures
    for jid, r in zip(ids, reqs):
        assert res[jid] == r["tokens"], f"request {jid}"
