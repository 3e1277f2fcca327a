"""A lattice database sharded over the ranks of a process group, one GPU per rank.

Each rank holds a contiguous slice of the rows with global ids (id_base = the slice's first row),
answers every query on its slice with the device search, and the ranks' answers -- k (id, distance)
pairs per query -- are all-gathered and merged by (distance, id). That gather is the path's only
exchange (NCCL over NVLink on the GPUs); the result on every rank equals the whole database's
exact answer.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


def shard_bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous split of n rows: the first n % world ranks take one row more."""
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def gather_merge(ids: torch.Tensor, dist_bits: torch.Tensor, merge: Callable, group=None):
    """All-gathers this rank's answer (ids [nq, k] int64, distances [nq, k] as int64 bit patterns of
    uint64) and merges the stacked [world, nq, k] answers with `merge(ids_all, dist_all)`."""
    world = dist.get_world_size(group)
    ids_all = [torch.empty_like(ids) for _ in range(world)]
    dist_all = [torch.empty_like(dist_bits) for _ in range(world)]
    dist.all_gather(ids_all, ids.contiguous(), group=group)
    dist.all_gather(dist_all, dist_bits.contiguous(), group=group)
    return merge(torch.stack(ids_all), torch.stack(dist_all))


def device_merge(ctx=None, stream: int = 0) -> Callable:
    """merge() for gather_merge on the GPU: the library's k-way merge kernel."""
    from . import knn_merge_device

    def merge(ids_all: torch.Tensor, dist_all: torch.Tensor):
        parts, nq, k = ids_all.shape
        out_i = torch.empty((nq, k), dtype=torch.int64, device=ids_all.device)
        out_d = torch.empty((nq, k), dtype=torch.int64, device=ids_all.device)
        knn_merge_device(ids_all.data_ptr(), dist_all.data_ptr(), parts, nq, k, out_i.data_ptr(), out_d.data_ptr(),
                         stream=stream, ctx=ctx)
        return out_i, out_d

    return merge
