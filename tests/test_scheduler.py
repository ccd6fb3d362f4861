"""Host scheduler logic (no GPU)."""
from types import SimpleNamespace

import pytest

from hayate_b200.config import EngineConfig
from hayate_b200.scheduler import SAMPLE, Scheduler, graph_bucket, graph_buckets


def req(i, n, max_tokens=4):
    return SimpleNamespace(id=i, prompt_tokens=list(range(n)), max_tokens=max_tokens, slot=-1,
                           _blocks=0, cache_pos=0, is_prefill=True, is_completed=False,
                           _last_launched=False)


def test_admission_is_fifo_and_bounded_by_slots_and_blocks():
    cfg = EngineConfig(max_num_seqs=3, max_batched_tokens=64, prefill_chunk=16, max_model_len=256)
    s = Scheduler(cfg, num_blocks=1 + 6, max_reqs=4)          # 6 usable blocks
    rs = [req(0, 30), req(1, 60), req(2, 5), req(3, 5)]
    s.waiting.extend(rs)
    got = s.admit()
    # r0 needs ceil(34/16)=3 blocks, r1 needs ceil(64/16)=4 > 3 left: FIFO stops there
    assert [r.id for r in got] == [0] and s.free_blocks == 3
    s.release(rs[0])
    got = s.admit()
    assert [r.id for r in got] == [1, 2, 3] and s.free_blocks == 0
    assert sorted(r.slot for r in got) == [0, 1, 2]
    s.waiting.append(req(4, 1))
    assert s.admit() == []                         # max_num_seqs reached


def test_schedule_decodes_first_then_chunked_prefill_within_budget():
    cfg = EngineConfig(max_num_seqs=8, max_batched_tokens=40, prefill_chunk=16, max_model_len=256)
    s = Scheduler(cfg, num_blocks=100, max_reqs=9)
    a, b, c = req(0, 50), req(1, 10), req(2, 7)
    s.waiting.extend([a, b, c])
    s.admit()
    c.is_prefill, c.cache_pos = False, 7           # c is decoding
    plan = s.schedule()
    assert [(e.req.id, e.start, e.q_len, e.flags) for e in plan.entries] == [
        (2, 7, 1, SAMPLE), (0, 0, 16, 0), (1, 0, 10, SAMPLE)]
    assert plan.num_tokens == 27 and plan.num_sample == 2 and not plan.decode_only
    a.cache_pos = 48
    plan = s.schedule()
    assert (plan.entries[1].start, plan.entries[1].q_len, plan.entries[1].flags) == (48, 2, SAMPLE)


def test_budget_cuts_prefill():
    cfg = EngineConfig(max_num_seqs=4, max_batched_tokens=8, prefill_chunk=16, max_model_len=256)
    s = Scheduler(cfg, num_blocks=100, max_reqs=5)
    s.waiting.extend([req(0, 30), req(1, 30)])
    s.admit()
    plan = s.schedule()
    assert [(e.req.id, e.q_len) for e in plan.entries] == [(0, 8)]


def test_request_checks():
    cfg = EngineConfig(max_num_seqs=4, max_batched_tokens=64, max_model_len=32)
    s = Scheduler(cfg, num_blocks=10, max_reqs=5)
    with pytest.raises(ValueError):
        s.check_request(req(0, 0))
    with pytest.raises(ValueError):
        s.check_request(req(1, 40))
    with pytest.raises(ValueError):
        EngineConfig(max_num_seqs=10, max_batched_tokens=4) and Scheduler(
            EngineConfig(max_num_seqs=10, max_batched_tokens=4), 10, 11)


def test_graph_buckets_cover_every_batch():
    bs = graph_buckets(256)
    assert bs[0] == 1 and bs[-1] == 256
    for n in range(1, 257):
        b = graph_bucket(n, 256)
        assert b >= n and b in bs


def test_output_is_capped_at_max_model_len():
    """A request whose max_tokens would run past max_model_len generates up to
    the length limit: its reservation covers exactly that many tokens."""
    cfg = EngineConfig(max_num_seqs=4, max_batched_tokens=64, max_model_len=64)
    s = Scheduler(cfg, num_blocks=20, max_reqs=5)
    long_out = req(0, 40, max_tokens=100)
    s.check_request(long_out)                       # admitted, not rejected
    assert s.token_limit(long_out) == 24
    assert s.reserve_for(long_out) == 4             # 64 tokens = 4 blocks
    short = req(1, 40, max_tokens=5)
    assert s.token_limit(short) == 5 and s.reserve_for(short) == 3
    edge = req(2, 63, max_tokens=0)                 # one token always, as the reference
    assert s.token_limit(edge) == 1 and s.reserve_for(edge) == 4
