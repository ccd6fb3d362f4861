"""Bit-exact numpy spec of the paged-KV bookkeeping -- TEST INFRASTRUCTURE ONLY.

The reference keeps one contiguous cache per request and rebuilds padded
batches every step (engine.py:80-194, qwen.py:66-106); it has no block pool,
slot mapping or block tables.  This module specifies them; the CUDA kernels in
``hayate_b200/csrc/pack.cu`` and the cache writes of ``qk_norm_rope.cu`` must
match it bit for bit.  Its link to the reference:

* positions: token j of a request with ``start`` cached tokens has position
  start + j, which equals the reference's position id for every real token
  (qwen.py:70-77: arange + cache_len - pad_len, the pad shift cancelling the
  left padding);
* cache contents: gathering a request's blocks in block-table order yields the
  reference's compacted per-request cache (engine.py:118-141).
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence

import numpy as np

BLOCK = 16


class PagedState:
    """Device-resident request state, mirrored on the host."""

    def __init__(self, max_reqs: int, tok_pitch: int, bt_pitch: int, num_blocks: int):
        self.req_tokens = np.zeros((max_reqs, tok_pitch), np.int32)
        self.block_tables = np.zeros((max_reqs, bt_pitch), np.int32)
        self.req_nblk = np.zeros(max_reqs, np.int32)
        # pops take the top: the first allocation returns block 0, then 1, ...
        self.free_stack = np.arange(num_blocks - 1, -1, -1, dtype=np.int32)
        self.free_top = num_blocks

    @property
    def num_blocks(self) -> int:
        return self.free_stack.shape[0]


def make_sched(slots: Sequence[int], starts: Sequence[int], qlens: Sequence[int],
               flags: Sequence[int]) -> np.ndarray:
    return np.array([list(slots), list(starts), list(qlens), list(flags)], np.int32)


def pack(st: PagedState, sched: np.ndarray, T: int) -> Dict[str, np.ndarray]:
    """One step: allocate blocks in schedule order, then emit the flat batch."""
    slots, starts, qlens, flags = (sched[i].astype(np.int64) for i in range(4))
    S = sched.shape[1]
    cu = np.zeros(S + 1, np.int32)
    cu[1:] = np.cumsum(qlens)
    assert cu[-1] == T, "schedule token count differs from T"
    top = st.free_top
    k = 0
    for i in range(S):
        s = int(slots[i])
        end = int(starts[i] + qlens[i])
        need = max(0, -(-end // BLOCK) - int(st.req_nblk[s]))
        for j in range(need):
            assert k < top, "block pool exhausted"
            st.block_tables[s, st.req_nblk[s] + j] = st.free_stack[top - 1 - k]
            k += 1
        st.req_nblk[s] += need
    st.free_top = top - k
    ids = np.zeros(T, np.int32)
    pos = np.zeros(T, np.int32)
    slot_map = np.zeros(T, np.int32)
    for i in range(S):
        s = int(slots[i])
        for j in range(int(qlens[i])):
            p = int(starts[i]) + j
            r = cu[i] + j
            ids[r] = st.req_tokens[s, p]
            pos[r] = p
            slot_map[r] = st.block_tables[s, p // BLOCK] * BLOCK + p % BLOCK
    samp = [i for i in range(S) if (flags[i] & 1) and qlens[i] > 0]
    return {
        "input_ids": ids, "positions": pos, "slot_mapping": slot_map, "cu_seqlens_q": cu,
        "seq_lens_k": (starts + qlens).astype(np.int32),
        "sample_rows": np.array([cu[i + 1] - 1 for i in samp], np.int32),
        "sample_seq": np.array(samp, np.int32),
    }


def commit(st: PagedState, next_tokens: np.ndarray, sample_seq: np.ndarray,
           sched: np.ndarray) -> None:
    for k, i in enumerate(sample_seq):
        s = sched[0, i]
        st.req_tokens[s, sched[1, i] + sched[2, i]] = next_tokens[k]


def free(st: PagedState, slots: Sequence[int], first: Optional[Sequence[int]] = None) -> None:
    """Blocks of each slot (from position first[i] on, if given) back onto the
    stack, slot by slot in list order, blocks in position order."""
    top = st.free_top
    for i, s in enumerate(slots):
        f = 0 if first is None else int(first[i])
        n = int(st.req_nblk[s]) - f
        st.free_stack[top:top + n] = st.block_tables[s, f:f + n]
        top += n
        st.req_nblk[s] = 0
    st.free_top = top


def push(st: PagedState, ids: Sequence[int]) -> None:
    """Block ids back onto the stack in list order (a prefix cache evicting)."""
    n = len(ids)
    st.free_stack[st.free_top:st.free_top + n] = np.asarray(ids, np.int32)
    st.free_top += n


def kv_append(cache_layer: np.ndarray, k: np.ndarray, v: np.ndarray,
              slot_mapping: np.ndarray) -> None:
    """cache_layer: [blocks][2][Hkv][16][D]; k, v: [T][Hkv][D]."""
    for t, s in enumerate(slot_mapping):
        if s < 0:
            continue
        b, j = divmod(int(s), BLOCK)
        cache_layer[b, 0, :, j] = k[t]
        cache_layer[b, 1, :, j] = v[t]


def gather(cache_layer: np.ndarray, bt_row: np.ndarray, n: int):
    """A request's first n cached tokens as contiguous (Hkv, n, D) K and V --
    the reference's per-request Cache layout of one layer (cache.py:7-10)."""
    nb = -(-n // BLOCK)
    blocks = cache_layer[bt_row[:nb]]                     # (nb, 2, Hkv, 16, D)
    k = np.concatenate(list(blocks[:, 0]), axis=1)[:, :n]
    v = np.concatenate(list(blocks[:, 1]), axis=1)[:, :n]
    return k, v
