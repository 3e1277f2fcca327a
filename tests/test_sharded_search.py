"""Sharded lattice search on world_size-2 gloo ranks (CPU): the shard split, global ids, the
all-gather of the ranks' answers and their merge give the whole database's exact answer. Each
rank's local search is the oracle here; on the GPUs it is the device search and the merge kernel."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from spatialdb_b200.sharded import gather_merge, shard_bounds


def test_shard_bounds_cover_rows():
    for n in (0, 1, 7, 10, 1000):
        for world in (1, 2, 3, 8):
            spans = [shard_bounds(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(h - l for l, h in spans) - min(h - l for l, h in spans) <= 1


def _rank(rank, world, port, db, q, k, out):
    import oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lo, hi = shard_bounds(db.shape[0], world, rank)
        ids, d = oracle.knn_l2(db[lo:hi], q, k, id_base=lo)

        def merge(ids_all, dist_all):
            mi, md = oracle.merge_topk(ids_all.numpy(), dist_all.numpy().view(np.uint64))
            return torch.from_numpy(mi), torch.from_numpy(md.view(np.int64))

        mi, md = gather_merge(torch.from_numpy(ids), torch.from_numpy(d.view(np.int64)), merge)
        out[rank] = (mi.numpy().copy(), md.numpy().view(np.uint64).copy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [1001, 7])
def test_two_ranks_match_whole_database(oracle, n):
    rng = np.random.default_rng(n)
    db = rng.integers(-1000, 1000, (n, 24)).astype(np.int64)
    db[n // 3] = db[n // 2]  # equal distances across shards
    q = rng.integers(-1000, 1000, (9, 24)).astype(np.int64)
    k = 10
    with mp.Manager() as m:
        out = m.dict()
        port = 29500 + (os.getpid() % 1000) + n % 7
        mp.spawn(_rank, args=(2, port, db, q, k, out), nprocs=2, join=True)
        res = dict(out)
    want_i, want_d = oracle.knn_l2(db, q, k)
    for r in range(2):
        np.testing.assert_array_equal(res[r][0], want_i)
        np.testing.assert_array_equal(res[r][1], want_d)
