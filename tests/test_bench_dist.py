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
