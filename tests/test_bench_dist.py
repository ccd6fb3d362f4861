"""The bench's multi-rank plumbing (barrier, max/sum over ranks) on gloo, CPU."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    bench.barrier(world, rank)
    # each rank times its own replica: value = all tokens / slowest rank's time
    ms = 100.0 + 50.0 * rank
    toks = 2560.0
    out[rank] = (bench.max_over_ranks(ms, world), bench.sum_over_ranks(toks, world))
    bench.barrier(world, rank)
    dist.destroy_process_group()


def test_two_rank_reductions_on_gloo():
    world = 2
    out = mp.Manager().dict()
    mp.spawn(_rank_main, args=(world, _free_port(), out), nprocs=world, join=True)
    assert out[0] == out[1] == (150.0, 5120.0)


def test_rank_shares_partition_the_request_set():
    """Each rank's share (computed alone, no communication) is its least-work
    part of the world x 256 request set: the shares are disjoint, cover the set,
    and their token loads differ by less than one request."""
    for world in (1, 2, 8):
        shares = [bench.rank_share(world, r) for r in range(world)]
        ids = [id(w) for s in shares for w in s]
        assert len(ids) == len(set(ids))
        prompts = sorted(tuple(w.prompt[:8]) + (len(w.prompt),) for s in shares for w in s)
        from hayate_b200.workloads import replicas
        allw = replicas(seed=0, n=bench.PER_GPU * world)
        assert prompts == sorted(tuple(w.prompt[:8]) + (len(w.prompt),) for w in allw)
        loads = [sum(len(w.prompt) + w.max_tokens for w in s) for s in shares]
        assert max(loads) - min(loads) <= bench.PROMPT_HI + bench.MAX_TOKENS
        assert all(w.max_tokens == 256 and 512 <= len(w.prompt) <= 4096 for s in shares for w in s)
