"""Prefix cache and the scheduler's block accounting with it (host only)."""
from types import SimpleNamespace

from hayate_b200.config import EngineConfig
from hayate_b200.prefix_cache import PrefixCache, block_hashes, cacheable_blocks
from hayate_b200.scheduler import Scheduler


def test_hash_chain_depends_on_everything_before():
    a = list(range(64))
    b = list(range(64))
    b[3] = 999                                  # differs in the first block only
    ha, hb = block_hashes(a, 16, 4), block_hashes(b, 16, 4)
    assert len(ha) == 4 and all(x != y for x, y in zip(ha, hb))
    c = a[:32] + [7] * 32                       # same first two blocks
    hc = block_hashes(c, 16, 4)
    assert hc[:2] == ha[:2] and hc[2:] != ha[2:]
    assert cacheable_blocks(33, 16) == 2 and cacheable_blocks(32, 16) == 1
    assert cacheable_blocks(1, 16) == 0


def test_match_acquire_offer_release_evict():
    c = PrefixCache()
    h = block_hashes(list(range(80)), 16, 5)
    assert c.match(h) == []
    assert c.offer(h[:3], [10, 11, 12]) == 3     # the offering request holds them
    assert c.match(h) == [10, 11, 12] and c.evictable == 0
    assert c.offer(h[2:5], [50, 13, 14]) == 0    # h[2] is held already: nothing taken
    c.acquire(h[:2])                             # a second request uses two of them
    c.release(h[:3])                             # the first one finishes
    assert c.evictable == 1                      # block 12: nobody references it
    assert c.evict(5) == [12] and c.match(h) == [10, 11]
    c.release(h[:2])
    assert sorted(c.evict(5)) == [10, 11] and c.held == 0


def _req(i, prompt, max_tokens=4):
    return SimpleNamespace(id=i, prompt_tokens=prompt, max_tokens=max_tokens, slot=-1,
                           _blocks=0, cache_pos=0, is_prefill=True, is_completed=False,
                           _last_launched=False)


def test_scheduler_takes_cached_prefix_and_counts_blocks():
    cfg = EngineConfig(max_num_seqs=8, max_batched_tokens=256, prefill_chunk=64,
                       max_model_len=1024, num_kv_blocks=40)
    cache = PrefixCache()
    sch = Scheduler(cfg, num_blocks=40, max_reqs=9, cache=cache)
    shared = list(range(100, 148))               # three full blocks
    a = _req(0, shared + [1, 2, 3])
    sch.waiting.append(a)
    assert sch.admit() == [a] and a._shared == 0
    need_a = a._blocks                           # ceil((51 + 4) / 16) = 4
    assert need_a == 4 and sch.free_blocks == 39 - 4
    # a's prefill wrote blocks 7, 8, 9 for its three full prompt blocks
    n = cacheable_blocks(len(a.prompt_tokens), 16)
    sch.offered(a, cache.offer(a._hashes[:n], [7, 8, 9]))
    assert a._shared == 3 and a._blocks == 1 and cache.held == 3
    b = _req(1, shared + [9, 9, 9, 9, 9])
    sch.waiting.append(b)
    assert sch.admit() == [b]
    assert b._shared_blocks == [7, 8, 9] and b.cache_pos == 48 and b._blocks == 1
    assert sch.free_blocks == 39 - 4 - 1
    sch.release(a)
    sch.release(b)
    assert sch.free_blocks == 39 - 3 and cache.evictable == 3   # the cache still holds 3
    # an admission short of room evicts idle cache blocks, oldest first: it needs
    # ceil(593 / 16) = 38 blocks with 36 free
    big = _req(2, list(range(500, 500 + 16 * 37)), max_tokens=1)
    sch.waiting.append(big)
    assert sch.admit() == [big]
    assert sch.take_evicted() == [7, 8] and sch.free_blocks == 0 and cache.held == 1
