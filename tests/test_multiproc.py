"""Replica mode across ranks (bench.py, torch.distributed over gloo on CPU):
each rank times its own replica; the job reports total tokens over the
max-over-ranks time.  The path itself has no collective (replicas only)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import bench
    w, r, _ = bench.dist_setup(None)
    assert (w, r) == (world, rank)
    # rank-dependent "elapsed ms": the job time is the slowest rank's
    mine = 100.0 + 10.0 * rank
    got = bench.max_over_ranks(mine, w, torch.device("cpu"))
    bench.barrier(w)
    out[rank] = got
    import torch.distributed as dist
    dist.destroy_process_group()


def test_max_over_ranks_gloo_world2():
    world = 2
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(world, _free_port(), out), nprocs=world, join=True)
    assert out[0] == out[1] == 110.0


def test_config_dict_reports_replicas():
    import bench
    c1, c4 = bench.config_dict(1), bench.config_dict(4)
    assert c1["parallelism"] == "single" and c4["parallelism"] == "replicas x4"
    assert c4["global_batch"] == 4 and c4["seq_len"] == bench.PROMPT + bench.GEN
