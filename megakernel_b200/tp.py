"""Tensor-parallel decode over NVLink (configs[4] mode b), host glue.

One process per GPU.  Every rank builds a ``MegakernelEngine`` with its
(rank, size); the ranks exchange the CUDA IPC handles of their exchange
buffers through ``torch.distributed`` (any backend; only host bytes move) and
map each other's buffers.  From then on the ranks make identical decode calls
and the kernels exchange data directly over NVLink: per layer each rank's
partial down projection (1024 fp32), per token every CTA's (max, index) pair.
The reference is single-GPU and has no counterpart.

``merge_partials`` / ``merge_argmax`` restate, on the host, what every rank's
kernel does with the exchanged values; the tests check them against the
single-GPU computation on CPU ranks.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from .bridge import MegakernelEngine


def split_range(total: int, rank: int, size: int) -> tuple[int, int]:
    """Rows [lo, hi) of a dimension of `total` owned by `rank` (even split)."""
    assert total % size == 0, (total, size)
    n = total // size
    return rank * n, (rank + 1) * n


def connect(engine: MegakernelEngine, group=None) -> None:
    """Exchange IPC handles over `group` and map every rank's buffer."""
    size = dist.get_world_size(group)
    assert size == engine.tp_size, (size, engine.tp_size)
    mine = engine.tp_ipc_handle()
    allh = [None] * size
    dist.all_gather_object(allh, mine, group=group)
    engine.tp_connect(allh)


def make_engine(flat, offsets, shape, device: int, group=None, **kw) -> MegakernelEngine:
    """A connected tensor-parallel engine for this process's rank of `group`."""
    rank, size = dist.get_rank(group), dist.get_world_size(group)
    eng = MegakernelEngine(flat=flat, offsets=offsets, shape=shape, device=device,
                           tp_rank=rank, tp_size=size, **kw)
    connect(eng, group)
    return eng


def merge_partials(x_after_attn: np.ndarray, partials: list[np.ndarray]) -> np.ndarray:
    """Layer output from the ranks' partial down projections: x' + sum_r p_r,
    added in rank order in fp32 (the kernel's order on every rank)."""
    v = x_after_attn.astype(np.float32).copy()
    for p in partials:
        v = (v + p.astype(np.float32)).astype(np.float32)
    return v


def merge_argmax(pairs: list[tuple[float, int]]) -> int:
    """Global greedy token from per-(rank, CTA) (max, index) pairs: the
    largest value, the lowest vocabulary index among equal values."""
    best_v, best_i = -np.inf, np.iinfo(np.int32).max
    for v, i in pairs:
        if v > best_v or (v == best_v and i < best_i):
            best_v, best_i = v, i
    return int(best_i)


def gather_logits(local: torch.Tensor, vocab: int, group=None) -> torch.Tensor:
    """Full logits rows from the ranks' captured slices ([n, vocab] fp32 on
    each rank, only its own vocab rows valid): an all-gather of the slices."""
    rank, size = dist.get_rank(group), dist.get_world_size(group)
    lo, hi = split_range(vocab, rank, size)
    mine = local[:, lo:hi].contiguous()
    parts = [torch.empty_like(mine) for _ in range(size)]
    dist.all_gather(parts, mine, group=group)
    return torch.cat(parts, dim=1)
