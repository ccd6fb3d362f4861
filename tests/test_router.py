"""Router over replica processes (CPU fakes; failures are made on the host)."""
import random

import pytest

from hayate_b200.router import Router
from router_fakes import fake_factory, fake_tokens


def _workload(n, seed=0):
    rng = random.Random(seed)
    return [([rng.randrange(1000) for _ in range(rng.randint(1, 40))], rng.randint(1, 12))
            for _ in range(n)]


def _run(router, work):
    ids = [router.submit(p, m) for p, m in work]
    res = router.wait_all(timeout=120)
    for jid, (p, m) in zip(ids, work):
        assert res[jid] == fake_tokens(p, m)
    return res


def test_router_spreads_work_and_returns_every_result():
    work = _workload(24)
    with Router(2, fake_factory) as r:
        _run(r, work)
        assert r.failures == []
        assert len({j.replica for j in r.jobs.values()}) == 2


@pytest.mark.parametrize("mode", ["exit", "hang"])
def test_router_requeues_work_of_a_failed_replica(mode):
    work = _workload(30, seed=1)
    with Router(3, fake_factory, {"failing_rank": 1, "fail": (mode, 3)},
                heartbeat_timeout=2.0) as r:
        _run(r, work)
        assert r.failures == [1]
        assert any(j.attempts > 1 for j in r.jobs.values())


def test_static_assignment_is_the_routers_rule_for_a_burst():
    """Jobs submitted together land where least_work_assignment puts them (the
    bench computes each rank's share with it, without communicating)."""
    from hayate_b200.router import least_work_assignment
    work = _workload(40, seed=3)
    with Router(3, fake_factory) as r:
        for p, m in work:
            r.submit(p, m)
        got = [r.jobs[j].replica for j in sorted(r.jobs)]
        r.wait_all(timeout=120)
    assert got == least_work_assignment([len(p) + m for p, m in work], 3)
    assert least_work_assignment([5, 1, 1, 1, 1, 1], 2) == [0, 1, 1, 1, 1, 1]
