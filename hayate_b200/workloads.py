"""Seeded synthetic workloads.

The reference benchmark builds prompts from random ASCII words and a tokenizer
(``benchmark.py:32-70``).  Neither the tokenizer nor a dataset exists offline, so
every workload here is token ids drawn uniformly from the vocabulary with fixed
seeds, in the shapes of the five benchmark configurations:

* ``single``     -- one 32-token prompt, 32 greedy tokens (fp32 parity case);
* ``upfront``    -- 10 requests, prompt lengths U[64,512], 256 tokens each, all
  submitted at once (the reference's "submit all upfront" mode,
  ``benchmark.py:204-236``);
* ``poisson``    -- 64 requests, exponential inter-arrival gaps of mean 20 ms,
  prompt lengths log-uniform in [128,2048], output lengths U[128,512] (a Poisson
  variant of "staggered arrivals", ``benchmark.py:239-303``);
* ``attn_micro`` -- the ragged attention operator case: 256 decode sequences
  with contexts log-uniform in [256,16384] plus 4 prefill chunks of 512 tokens
  with prior contexts {0, 512, 1536, 3584};
* ``replicas``   -- 2048 requests, prompt lengths U[512,4096], 256 tokens each;
  ``replica_share`` is one GPU's part of the N x 256-request version of it,
  split by the router's least-outstanding-work rule.
"""
from __future__ import annotations

import math
import random
from dataclasses import dataclass, field
from typing import List

import numpy as np
import torch

VOCAB = 151_936


@dataclass
class SyntheticRequest:
    prompt: List[int]
    max_tokens: int
    arrival_s: float = 0.0


def _ids(gen: torch.Generator, n: int, vocab: int) -> List[int]:
    return torch.randint(0, vocab, (n,), generator=gen, dtype=torch.int64).tolist()


def single(seed: int = 0, vocab: int = VOCAB, prompt_len: int = 32,
           max_tokens: int = 32) -> List[SyntheticRequest]:
    g = torch.Generator().manual_seed(seed)
    return [SyntheticRequest(_ids(g, prompt_len, vocab), max_tokens)]


def upfront(seed: int = 0, vocab: int = VOCAB, n: int = 10, lo: int = 64, hi: int = 512,
            max_tokens: int = 256) -> List[SyntheticRequest]:
    rng = random.Random(seed)
    lens = [rng.randint(lo, hi) for _ in range(n)]
    g = torch.Generator().manual_seed(seed)
    return [SyntheticRequest(_ids(g, L, vocab), max_tokens) for L in lens]


def poisson(seed: int = 0, vocab: int = VOCAB, n: int = 64, mean_gap_s: float = 0.020,
            lo: int = 128, hi: int = 2048, out_lo: int = 128,
            out_hi: int = 512) -> List[SyntheticRequest]:
    rng = random.Random(seed)
    g = torch.Generator().manual_seed(seed)
    t = 0.0
    reqs = []
    for i in range(n):
        if i > 0:
            t += rng.expovariate(1.0 / mean_gap_s)
        L = int(round(math.exp(rng.uniform(math.log(lo), math.log(hi)))))
        out = rng.randint(out_lo, out_hi)
        reqs.append(SyntheticRequest(_ids(g, L, vocab), out, arrival_s=t))
    return reqs


def replicas(seed: int = 0, vocab: int = VOCAB, n: int = 2048, lo: int = 512,
             hi: int = 4096, max_tokens: int = 256) -> List[SyntheticRequest]:
    rng = random.Random(seed)
    lens = [rng.randint(lo, hi) for _ in range(n)]
    g = torch.Generator().manual_seed(seed)
    return [SyntheticRequest(_ids(g, L, vocab), max_tokens) for L in lens]


REPLICA_PER_GPU = 256


def replica_share(world: int, rank: int, seed: int = 0,
                  per_gpu: int = REPLICA_PER_GPU) -> List[SyntheticRequest]:
    """Rank ``rank``'s requests of the ``world * per_gpu`` replica workload
    (prompts U[512,4096], 256 tokens), assigned as the router assigns requests
    that arrive together (least outstanding work); the same on every rank, so
    no communication is needed.  At world=8 the set is the 2048-request one."""
    from .router import least_work_assignment
    ws = replicas(seed=seed, n=per_gpu * world)
    owner = least_work_assignment([len(w.prompt) + w.max_tokens for w in ws], world)
    return [w for w, o in zip(ws, owner) if o == rank]


@dataclass
class AttnMicro:
    """Shapes of the ragged attention operator case (one layer)."""
    decode_ctx: List[int]
    prefill_prior: List[int] = field(default_factory=lambda: [0, 512, 1536, 3584])
    prefill_len: int = 512

    @property
    def num_seqs(self) -> int:
        return len(self.decode_ctx) + len(self.prefill_prior)

    def seq_lens_k(self) -> List[int]:
        return [p + self.prefill_len for p in self.prefill_prior] + list(self.decode_ctx)

    def q_lens(self) -> List[int]:
        return [self.prefill_len] * len(self.prefill_prior) + [1] * len(self.decode_ctx)


def attn_micro(seed: int = 0, n_decode: int = 256, lo: int = 256,
               hi: int = 16384) -> AttnMicro:
    rng = np.random.default_rng(seed)
    ctx = np.round(np.exp(rng.uniform(math.log(lo), math.log(hi), size=n_decode))).astype(int)
    return AttnMicro(decode_ctx=[int(c) for c in ctx])
