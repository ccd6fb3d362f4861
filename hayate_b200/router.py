"""Request-level data parallelism: one engine replica per GPU behind a router.

The step does not shard below the request: every request's tokens, KV blocks
and attention live on one GPU.  N GPUs therefore run N independent replicas
(one OS process each, no collective on the data path), and this router hands
requests to them:

* assignment: least outstanding work, measured as prompt + max_tokens tokens
  not yet finished on the replica (long prompts spread evenly);
* failure detection on the host: a replica whose process exits, or whose
  heartbeat stops for ``heartbeat_timeout`` seconds, is marked dead and every
  request it had not finished is re-queued on the live replicas.  Results are
  deterministic per request (greedy decoding), so a re-run request returns the
  tokens it would have returned the first time.

The replica body is ``engine_factory(rank) -> engine`` (an object with the
``Engine`` surface: ``add_request``, ``generate``); the default builds a
``hayate_b200.engine.Engine`` on ``cuda:rank``.  Tests pass CPU fakes.
"""
from __future__ import annotations

import multiprocessing as mp
import queue
import time
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional

STOP = "__stop__"


@dataclass
class Job:
    id: int
    prompt: List[int]
    max_tokens: int
    replica: int = -1
    attempts: int = 0


def least_work_assignment(costs: List[int], n: int) -> List[int]:
    """Replica of each job when jobs of these costs (prompt + max_tokens tokens)
    arrive together: each goes, in order, to the replica with the least
    outstanding work so far (the lowest index on ties) -- ``Router._assign``'s
    rule before any job has finished.  Deterministic, so every rank of a
    multi-process run can compute its own share without communicating."""
    load = [0] * n
    out = []
    for c in costs:
        r = min(range(n), key=lambda k: load[k])
        out.append(r)
        load[r] += c
    return out


def default_engine_factory(rank: int, **engine_kwargs):
    import torch
    from .engine import Engine
    torch.cuda.set_device(rank)
    return Engine(device=f"cuda:{rank}", **engine_kwargs)


def _replica_main(rank, factory, factory_kwargs, in_q, out_q, heartbeat):
    """Replica process: feed requests into the engine, step it, report results."""
    from .engine import Request
    eng = factory(rank, **factory_kwargs)
    capture = getattr(eng, "capture_graphs", None)
    if capture is not None:              # decode graphs for every batch size, before timing
        capture()
    live: Dict[int, object] = {}
    heartbeat[rank] = time.time()
    out_q.put(("ready", rank, None, None))
    while True:
        try:                             # never block while requests are in flight
            msg = in_q.get_nowait() if live else in_q.get(timeout=0.5)
        except queue.Empty:
            msg = None
        while msg is not None:
            if msg == STOP:
                out_q.put(("stopped", rank, None, None))
                return
            jid, prompt, max_tokens = msg
            req = Request(id=jid, prompt=prompt, max_tokens=max_tokens)
            eng.add_request(req)
            live[jid] = req
            try:
                msg = in_q.get_nowait()
            except queue.Empty:
                msg = None
        if live:
            eng.generate()
            for jid in [j for j, r in live.items() if r.is_completed]:
                out_q.put(("done", rank, jid, list(live.pop(jid).tokens)))
        heartbeat[rank] = time.time()


class Router:
    def __init__(self, n_replicas: int, engine_factory: Callable = default_engine_factory,
                 factory_kwargs: Optional[dict] = None, heartbeat_timeout: float = 60.0,
                 start_method: str = "spawn"):
        self.n = n_replicas
        self.ctx = mp.get_context(start_method)
        self.heartbeat = self.ctx.Array("d", [0.0] * n_replicas)
        self.out_q = self.ctx.Queue()
        self.in_qs = [self.ctx.Queue() for _ in range(n_replicas)]
        self.procs = [self.ctx.Process(target=_replica_main, daemon=True,
                                       args=(r, engine_factory, factory_kwargs or {},
                                             self.in_qs[r], self.out_q, self.heartbeat))
                      for r in range(n_replicas)]
        self.hb_timeout = heartbeat_timeout
        self.jobs: Dict[int, Job] = {}
        self.results: Dict[int, List[int]] = {}
        self.load = [0] * n_replicas
        self.alive = [True] * n_replicas
        self.ready = [False] * n_replicas
        self.failures: List[int] = []
        self._next_id = 0
        for p in self.procs:
            p.start()

    # ------------------------------------------------------------ submission
    def submit(self, prompt: List[int], max_tokens: int) -> int:
        jid = self._next_id
        self._next_id += 1
        self.jobs[jid] = Job(jid, list(prompt), max_tokens)
        self._assign(self.jobs[jid])
        return jid

    def _assign(self, job: Job) -> None:
        live = [r for r in range(self.n) if self.alive[r]]
        if not live:
            raise RuntimeError("no live replica left")
        r = min(live, key=lambda k: self.load[k])
        job.replica = r
        job.attempts += 1
        self.load[r] += len(job.prompt) + job.max_tokens
        self.in_qs[r].put((job.id, job.prompt, job.max_tokens))

    # ------------------------------------------------------------ progress
    def _mark_dead(self, r: int) -> None:
        if not self.alive[r]:
            return
        self.alive[r] = False
        self.failures.append(r)
        self.load[r] = 0
        for job in self.jobs.values():
            if job.replica == r and job.id not in self.results:
                self._assign(job)

    def _check_health(self) -> None:
        now = time.time()
        for r in range(self.n):
            if not self.alive[r]:
                continue
            p = self.procs[r]
            if p.exitcode is not None:
                self._mark_dead(r)
            elif self.ready[r] and now - self.heartbeat[r] > self.hb_timeout:
                p.kill()
                self._mark_dead(r)

    def poll(self, timeout: float = 0.1) -> int:
        """Collect finished results; returns how many arrived."""
        n = 0
        deadline = time.time() + timeout
        while True:
            try:
                kind, r, jid, toks = self.out_q.get(timeout=max(0.0, deadline - time.time()))
            except queue.Empty:
                break
            if kind == "ready":
                self.ready[r] = True
            elif kind == "done" and jid not in self.results and self.alive[r]:
                self.results[jid] = toks
                job = self.jobs[jid]
                self.load[r] -= len(job.prompt) + job.max_tokens
                n += 1
        self._check_health()
        return n

    def wait_all(self, timeout: float = 3600.0) -> Dict[int, List[int]]:
        end = time.time() + timeout
        while len(self.results) < len(self.jobs):
            if time.time() > end:
                raise TimeoutError(f"{len(self.jobs) - len(self.results)} requests unfinished")
            self.poll(0.2)
        return dict(self.results)

    def close(self) -> None:
        for r in range(self.n):
            if self.alive[r] and self.procs[r].is_alive():
                self.in_qs[r].put(STOP)
        for p in self.procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
                p.join(timeout=5)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
