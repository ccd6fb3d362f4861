"""CPU stand-ins for the router tests (importable by spawned replica processes)."""
import os
import time

from hayate_b200.engine import Request  # noqa: F401  (the replica builds these)


def fake_tokens(prompt, max_tokens):
    """Deterministic 'greedy' output of the fake engine."""
    s = sum(prompt)
    return [(s * 31 + 7 * i) % 1000 for i in range(max(max_tokens, 1))]


class FakeEngine:
    """The Engine surface (add_request / generate) over fake_tokens, one token per
    request per step.  ``fail`` = ("exit", n) exits the process at step n,
    ("hang", n) stops making progress (and heartbeats) at step n."""

    def __init__(self, rank, fail=None):
        self.rank = rank
        self.fail = fail
        self.reqs = []
        self.steps = 0

    def add_request(self, r):
        self.reqs.append(r)

    def generate(self):
        self.steps += 1
        if self.fail is not None and self.steps >= self.fail[1]:
            if self.fail[0] == "exit":
                os._exit(3)
            while True:                      # host-side hang
                time.sleep(1)
        live = [r for r in self.reqs if not r.is_completed]
        for r in live:
            want = fake_tokens(r.prompt, r.max_tokens)
            r.tokens.append(want[len(r.tokens)])
            if len(r.tokens) >= r.max_tokens:
                r.is_completed = True
        self.reqs = [r for r in self.reqs if not r.is_completed]
        return bool(live)


def fake_factory(rank, failing_rank=None, fail=None):
    return FakeEngine(rank, fail if rank == failing_rank else None)
