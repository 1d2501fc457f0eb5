"""Host-side restatement of the tensor-parallel exchange (megakernel_b200.tp)
on CPU ranks (gloo, world 2): each rank computes its slice of the MLP and of
the LM head of one decode step; the merged result equals the single-device
computation, and every rank picks the same token."""
import os
import socket

import numpy as np
import torch
import torch.multiprocessing as mp

from megakernel_b200 import tp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _problem(seed=0, H=64, I=192, V=512):
    g = np.random.default_rng(seed)
    x = g.standard_normal(H).astype(np.float32)
    wg = (0.1 * g.standard_normal((I, H))).astype(np.float32)
    wu = (0.1 * g.standard_normal((I, H))).astype(np.float32)
    wd = (0.1 * g.standard_normal((H, I))).astype(np.float32)
    emb = g.standard_normal((V, H)).astype(np.float32)
    emb[7] = emb[300] = emb[5] + 0.0  # exact ties: lowest index must win
    return x, wg, wu, wd, emb


def _mlp(x, wg, wu, wd):
    gt, up = wg @ x, wu @ x
    return wd @ ((gt / (1 + np.exp(-gt))) * up)


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world)
    x, wg, wu, wd, emb = _problem()
    lo, hi = tp.split_range(wg.shape[0], rank, world)
    part = _mlp(x, wg[lo:hi], wu[lo:hi], wd[:, lo:hi]).astype(np.float32)
    parts = [torch.empty(x.shape[0]) for _ in range(world)]
    dist.all_gather(parts, torch.from_numpy(part))
    xo = tp.merge_partials(x, [p.numpy() for p in parts])
    v0, v1 = tp.split_range(emb.shape[0], rank, world)
    lg = emb[v0:v1] @ (xo / np.sqrt((xo * xo).mean() + 1e-6))
    i = int(np.argmax(lg))
    pairs = [None] * world
    dist.all_gather_object(pairs, (float(lg[i]), v0 + i))
    out[rank] = (xo, tp.merge_argmax(pairs))
    dist.destroy_process_group()


def test_tp_merge_matches_single_device_gloo_world2():
    world = 2
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(world, _free_port(), out), nprocs=world, join=True)
    x, wg, wu, wd, emb = _problem()
    want = x + _mlp(x, wg, wu, wd)
    (x0, t0), (x1, t1) = out[0], out[1]
    assert np.array_equal(x0, x1) and t0 == t1
    assert np.abs(x0 - want).max() < 1e-4
    ref = emb @ (want / np.sqrt((want * want).mean() + 1e-6))
    assert t0 == int(np.argmax(ref))


def test_merge_argmax_lowest_index_on_ties():
    assert tp.merge_argmax([(1.0, 9), (2.0, 40), (2.0, 3), (0.5, 1)]) == 3
    assert tp.split_range(151936, 7, 8) == (132944, 151936)
