"""Prefix caching over the paged KV blocks (host side).

The reference lists prefix caching as future work (README.md:70); nothing on
its path shares KV between requests.  Here a full 16-token block of a prompt is
identified by a hash chain over the prompt's blocks up to and including it, so
two prompts that share their first k full blocks share the first k chain
hashes, and the KV those blocks hold (keys and values of a token depend only on
the tokens before it) can serve both.

The cache holds physical block ids.  A request admitted with a cached prefix
takes a reference on each of its blocks and starts its prefill after them; when
its prefill is done, its own full prompt blocks are offered to the cache, which
keeps each one whose hash it does not hold yet (the request's reference on it
moves to the cache).  A finished request drops its references; blocks nobody
references stay cached, least recently used first out, until the engine needs
their room and evicts them back to the device pool.
"""
from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass
from typing import Dict, List, Sequence


def block_hashes(tokens: Sequence[int], block_size: int, limit: int) -> List[int]:
    """Chain hashes of the first ``limit`` full blocks of ``tokens``."""
    out, h = [], 0
    n = min(limit, len(tokens) // block_size)
    for b in range(n):
        h = hash((h, tuple(int(t) for t in tokens[b * block_size:(b + 1) * block_size])))
        out.append(h)
    return out


def cacheable_blocks(prompt_len: int, block_size: int) -> int:
    """Full prompt blocks a request may take from (or give to) the cache: at
    least the last prompt token is always computed, to produce the first token."""
    return max(0, (prompt_len - 1) // block_size)


@dataclass
class _Entry:
    block: int
    refs: int


class PrefixCache:
    def __init__(self) -> None:
        self._entries: Dict[int, _Entry] = {}
        self._idle: "OrderedDict[int, None]" = OrderedDict()   # refs == 0, oldest first

    def __len__(self) -> int:
        return len(self._entries)

    @property
    def held(self) -> int:
        """Blocks the cache holds (referenced or not)."""
        return len(self._entries)

    @property
    def evictable(self) -> int:
        return len(self._idle)

    def match(self, hashes: Sequence[int]) -> List[int]:
        """Block ids of the longest cached prefix of ``hashes``."""
        out = []
        for h in hashes:
            e = self._entries.get(h)
            if e is None:
                break
            out.append(e.block)
        return out

    def acquire(self, hashes: Sequence[int]) -> None:
        for h in hashes:
            e = self._entries[h]
            if e.refs == 0:
                self._idle.pop(h, None)
            e.refs += 1

    def release(self, hashes: Sequence[int]) -> None:
        for h in hashes:
            e = self._entries[h]
            e.refs -= 1
            if e.refs == 0:
                self._idle[h] = None

    def offer(self, hashes: Sequence[int], blocks: Sequence[int]) -> int:
        """Take the blocks of a request's prompt (hash i held in block i), from the
        first on, until a hash the cache already holds; each taken block keeps one
        reference for the offering request.  Returns how many were taken."""
        n = 0
        for h, b in zip(hashes, blocks):
            if h in self._entries:
                break
            self._entries[h] = _Entry(int(b), 1)
            n += 1
        return n

    def evict(self, n: int) -> List[int]:
        """Drop up to ``n`` unreferenced blocks, least recently released first;
        returns their ids (to go back to the device pool)."""
        out = []
        while self._idle and len(out) < n:
            h, _ = self._idle.popitem(last=False)
            out.append(self._entries.pop(h).block)
        return out
