"""Host-side continuous-batching scheduler (pure Python, no device calls).

Replaces the reference's step policy (hayate/engine/engine.py:196-217): FIFO
admission, then every step one *mixed* batch -- all running decodes (one token
each) followed by prefill chunks of at most ``prefill_chunk`` tokens -- within a
``max_batched_tokens`` budget.  The reference instead runs padded prefill
groups of 8 and a separate decode forward.

Admission reserves a request's worst-case KV blocks (prompt + max_tokens) so
the device block pool can never run dry mid-flight; no preemption is needed.
A request generates at most ``max_model_len - len(prompt)`` tokens: one whose
``max_tokens`` would take it past ``max_model_len`` completes there (its token
row and block table are sized by that length), as a length-capped request.
Slot ``max_reqs - 1`` is kept for the padding rows of CUDA-graph batches.

With a prefix cache, a request first takes the longest cached prefix of its
prompt's full blocks (its prefill then starts after them) and reserves only the
rest; blocks the cache holds are not free, and unreferenced ones are evicted
(oldest first) when an admission needs their room.  The scheduler only counts;
the engine moves the evicted block ids back to the device pool.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field
from typing import Deque, List, Optional, Tuple

from .config import EngineConfig
from .prefix_cache import PrefixCache, block_hashes, cacheable_blocks

# sched flags
SAMPLE = 1


@dataclass
class StepEntry:
    req: object          # the engine's Request
    start: int           # tokens already in the KV cache
    q_len: int           # tokens computed this step
    flags: int           # SAMPLE if the last row yields a token


@dataclass
class StepPlan:
    entries: List[StepEntry] = field(default_factory=list)

    @property
    def num_seqs(self) -> int:
        return len(self.entries)

    @property
    def num_tokens(self) -> int:
        return sum(e.q_len for e in self.entries)

    @property
    def num_sample(self) -> int:
        return sum(1 for e in self.entries if e.flags & SAMPLE)

    @property
    def decode_only(self) -> bool:
        return all(e.q_len == 1 and e.start > 0 for e in self.entries)


def blocks_for(tokens: int, block_size: int) -> int:
    return -(-tokens // block_size)


class Scheduler:
    def __init__(self, cfg: EngineConfig, num_blocks: int, max_reqs: int,
                 cache: Optional[PrefixCache] = None):
        if cfg.max_num_seqs > cfg.max_batched_tokens:
            raise ValueError("max_num_seqs must not exceed max_batched_tokens")
        self.cfg = cfg
        self.pad_slot = max_reqs - 1
        self.free_slots: Deque[int] = deque(range(max_reqs - 1))
        self.total_blocks = num_blocks - 1         # one block for the padding slot
        self.free_blocks = self.total_blocks
        self.waiting: Deque = deque()
        self.running: List = []
        self.cache = cache
        self.evicted: List[int] = []               # cache blocks for the device pool

    # ---------------------------------------------------------------- admission
    def token_limit(self, req) -> int:
        """Tokens the request generates at most: its max_tokens (at least one, as
        the reference's prefill always samples one), capped so that prompt plus
        output stay within max_model_len."""
        return min(max(req.max_tokens, 1), self.cfg.max_model_len - len(req.prompt_tokens))

    def reserve_for(self, req) -> int:
        return blocks_for(len(req.prompt_tokens) + self.token_limit(req), self.cfg.block_size)

    def check_request(self, req) -> None:
        n = len(req.prompt_tokens)
        if n == 0:
            raise ValueError(f"request {req.id}: empty prompt")
        if n + 1 > self.cfg.max_model_len:
            raise ValueError(f"request {req.id}: prompt of {n} tokens exceeds max_model_len "
                             f"{self.cfg.max_model_len}")
        if self.reserve_for(req) > self.total_blocks:
            raise ValueError(f"request {req.id}: needs more KV blocks than the cache holds")

    def admit(self) -> List:
        """Move waiting requests into the running set (FIFO, stop at the first misfit)."""
        admitted = []
        while self.waiting and len(self.running) < self.cfg.max_num_seqs and self.free_slots:
            req = self.waiting[0]
            hashes, shared = [], []
            if self.cache is not None:
                bs = self.cfg.block_size
                hashes = block_hashes(req.prompt_tokens, bs,
                                      cacheable_blocks(len(req.prompt_tokens), bs))
                shared = self.cache.match(hashes)
            need = self.reserve_for(req) - len(shared)
            if need > self.free_blocks and self.cache is not None:
                # evict idle cache blocks, never those this request is about to use
                self.cache.acquire(hashes[:len(shared)])
                got = self.cache.evict(need - self.free_blocks)
                self.cache.release(hashes[:len(shared)])
                self.evicted += got
                self.free_blocks += len(got)
            if need > self.free_blocks:
                break
            self.waiting.popleft()
            req.slot = self.free_slots.popleft()
            req._blocks = need
            req._hashes = hashes
            req._shared_blocks = list(shared)       # adopted cache blocks, in order
            req._shared = len(shared)               # leading blocks the cache holds
            if shared:
                self.cache.acquire(hashes[:len(shared)])
                req.cache_pos = len(shared) * self.cfg.block_size
            self.free_blocks -= need
            self.running.append(req)
            admitted.append(req)
        return admitted

    def offered(self, req, n: int) -> None:
        """n more of the request's prompt blocks now belong to the cache."""
        req._shared += n
        req._blocks -= n

    def release(self, req) -> None:
        self.running.remove(req)
        self.free_slots.append(req.slot)
        self.free_blocks += req._blocks
        req._blocks = 0
        if self.cache is not None and req._shared:
            self.cache.release(req._hashes[:req._shared])

    def take_evicted(self) -> List[int]:
        out, self.evicted = self.evicted, []
        return out

    # ---------------------------------------------------------------- one step
    def schedule(self) -> StepPlan:
        budget = self.cfg.max_batched_tokens
        plan = StepPlan()
        for r in self.running:                      # decodes first, one token each
            if not r.is_prefill and not r.is_completed and not r._last_launched:
                plan.entries.append(StepEntry(r, r.cache_pos, 1, SAMPLE))
                budget -= 1
        for r in self.running:                      # then prefill chunks, FIFO
            if not r.is_prefill or budget <= 0:
                continue
            rem = len(r.prompt_tokens) - r.cache_pos
            q = min(rem, self.cfg.prefill_chunk, budget)
            if q <= 0:
                continue
            done = r.cache_pos + q == len(r.prompt_tokens)
            plan.entries.append(StepEntry(r, r.cache_pos, q, SAMPLE if done else 0))
            budget -= q
        return plan


def graph_bucket(n: int, max_seqs: int) -> int:
    """Smallest captured batch size holding n decode rows."""
    b = 1
    while b < n:
        b = b * 2 if b < 16 else b + 16
    return min(b, max_seqs)


def graph_buckets(max_seqs: int) -> List[int]:
    out, b = [], 1
    while b < max_seqs:
        out.append(b)
        b = b * 2 if b < 16 else b + 16
    out.append(max_seqs)
    return out
