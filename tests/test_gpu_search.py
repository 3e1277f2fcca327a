"""Parity of the device lattice k-NN search with the oracle's exact brute force.

Inputs are the embed+search workload's distribution (Gaussian-mixture embeddings, L2-normalized,
quantized with VocabLattice's options) at sizes the oracle finishes in seconds, plus the edge cases:
ragged dimensions, k at its limits, databases smaller than k, empty databases, duplicate rows (equal
distances), data the tensor-core bound cannot decide, components outside int32, sharded databases
merged on the device.
"""
import ctypes

import numpy as np
import pytest

import spatialdb_b200 as slx
from spatialdb_b200 import synth

pytestmark = pytest.mark.gpu

OPT = slx.VOCAB_LATTICE_OPTIONS


@pytest.fixture(scope="module")
def ctx():
    return slx.Context(0)


def _ref(oracle, db, q, k, opt=OPT, id_base=0):
    dq = oracle.quantize_dense(db, opt.zero_threshold, opt.global_scale)
    qq = oracle.quantize_dense(q, opt.zero_threshold, opt.global_scale)
    return oracle.knn_l2(dq, qq, k, id_base)


def _check(lat, oracle, db, q, k, exact=False, opt=OPT, id_base=0):
    ids, dist = lat.query_k_nearest_l2(q, k, exact=exact)
    rid, rdist = _ref(oracle, db, q, k, opt, id_base)
    np.testing.assert_array_equal(dist, rdist)
    np.testing.assert_array_equal(ids, rid)
    return lat.last_exact


@pytest.mark.parametrize("n,dim,nq,k", [(20000, 768, 300, 10), (5000, 384, 200, 1), (3000, 100, 130, 16),
                                        (777, 1000, 64, 7)])
def test_mixture_matches_oracle(ctx, oracle, n, dim, nq, k):
    rng = np.random.default_rng(n + dim)
    c = synth.mixture_centres(rng, dim, 64)
    db = synth.gaussian_mixture(rng, n, dim, centre_vectors=c)
    q = synth.gaussian_mixture(rng, nq, dim, centre_vectors=c)
    lat = slx.EmbeddingLattice(db, ctx=ctx)
    fell_back = _check(lat, oracle, db, q, k)
    assert fell_back <= nq // 10, f"{fell_back} of {nq} queries needed the exact scan"
    assert _check(lat, oracle, db, q[:50], k, exact=True) == 50


def test_small_database_pads(ctx, oracle):
    rng = np.random.default_rng(1)
    db = synth.gaussian_mixture(rng, 5, 64, centres=4)
    q = synth.gaussian_mixture(rng, 3, 64, centres=4)
    lat = slx.EmbeddingLattice(db, ctx=ctx)
    ids, dist = lat.query_k_nearest_l2(q, 10)
    assert (ids[:, 5:] == -1).all() and (dist[:, 5:] == np.iinfo(np.uint64).max).all()
    _check(lat, oracle, db, q, 10)
    ids0, _ = lat.query_k_nearest_l2(q, 0)
    assert ids0.shape == (3, 0)


def test_empty_database(ctx):
    lat = slx.EmbeddingLattice(np.zeros((0, 32), np.float32), ctx=ctx)
    ids, dist = lat.query_k_nearest_l2(np.ones((2, 32), np.float32) / 8, 4)
    assert (ids == -1).all() and (dist == np.iinfo(np.uint64).max).all()


def test_duplicate_rows_order_by_id(ctx, oracle):
    """Equal distances: every row appears three times; the answer lists equal distances by id, and
    the bound cannot separate the copies, so those queries take the exact scan."""
    rng = np.random.default_rng(2)
    base = synth.gaussian_mixture(rng, 700, 128, centres=8)
    db = np.concatenate([base, base, base])
    q = np.concatenate([base[:40], synth.gaussian_mixture(rng, 40, 128, centres=8)])
    lat = slx.EmbeddingLattice(db, ctx=ctx)
    _check(lat, oracle, db, q, 16)
    _check(lat, oracle, db, q, 3)


def test_large_norms_take_exact_scan(ctx, oracle):
    """|q| + |d| >= 2^31 (global scale 2e9 on unit vectors): the bound's key arithmetic could overflow,
    so every query is answered by the exact scan -- same answer."""
    rng = np.random.default_rng(3)
    opt = slx.QuantizationOptions(0.001, 2_000_000_000)
    db = synth.gaussian_mixture(rng, 2000, 256, centres=16)
    q = synth.gaussian_mixture(rng, 50, 256, centres=16)
    lat = slx.EmbeddingLattice(db, opt, ctx=ctx)
    assert _check(lat, oracle, db, q, 10, opt=opt) == 50


def test_zero_threshold_and_sparse_rows(ctx, oracle):
    """Components below the threshold are zero (EmbeddingAdapter.Quantize drops them); rows with few
    surviving components and all-zero rows."""
    rng = np.random.default_rng(4)
    db = rng.standard_normal((1500, 96)).astype(np.float32) * 0.01
    db[::7] = 0
    q = rng.standard_normal((40, 96)).astype(np.float32) * 0.01
    opt = slx.QuantizationOptions(0.008, 1_000_000_000)
    lat = slx.EmbeddingLattice(db, opt, ctx=ctx)
    _check(lat, oracle, db, q, 12, opt=opt)


def test_out_of_int32_is_range_error(ctx):
    db = np.full((4, 16), 0.5, np.float32)
    with pytest.raises(slx.IndexOutOfRangeError):
        slx.EmbeddingLattice(db, slx.QuantizationOptions(0.0, 10_000_000_000), ctx=ctx)
    bad = db.copy()
    bad[1, 3] = np.nan  # (long)NaN = long.MinValue
    with pytest.raises(slx.IndexOutOfRangeError):
        slx.EmbeddingLattice(bad, ctx=ctx)
    lat = slx.EmbeddingLattice(db, ctx=ctx)
    with pytest.raises(slx.IndexOutOfRangeError):
        lat.query_k_nearest_l2(np.full((1, 16), 3.0, np.float32), 2)
    with pytest.raises(slx.SlxError):
        lat.query_k_nearest_l2(db[:1], 17)


def test_sharded_merge_matches_whole(ctx, oracle):
    """Shards carry global ids (id_base); their answers, stacked [parts][nq][k], merge on the device
    into the whole database's answer."""
    import torch

    rng = np.random.default_rng(5)
    c = synth.mixture_centres(rng, 192, 32)
    db = synth.gaussian_mixture(rng, 9000, 192, centre_vectors=c)
    q = synth.gaussian_mixture(rng, 100, 192, centre_vectors=c)
    k, parts = 10, 3
    bounds = [0, 2500, 6100, 9000]
    ids = np.empty((parts, 100, k), np.int64)
    dist = np.empty((parts, 100, k), np.uint64)
    for p in range(parts):
        lat = slx.EmbeddingLattice(db[bounds[p]:bounds[p + 1]], id_base=bounds[p], ctx=ctx)
        ids[p], dist[p] = lat.query_k_nearest_l2(q, k)
        lat.close()
    d_ids = torch.from_numpy(ids).cuda()
    d_dist = torch.from_numpy(dist.view(np.int64)).cuda()
    o_ids = torch.empty((100, k), dtype=torch.int64, device="cuda")
    o_dist = torch.empty((100, k), dtype=torch.int64, device="cuda")
    slx.knn_merge_device(d_ids.data_ptr(), d_dist.data_ptr(), parts, 100, k, o_ids.data_ptr(), o_dist.data_ptr(),
                         stream=torch.cuda.current_stream().cuda_stream, ctx=ctx)
    torch.cuda.synchronize()
    rid, rdist = _ref(oracle, db, q, k)
    np.testing.assert_array_equal(o_dist.cpu().numpy().view(np.uint64), rdist)
    np.testing.assert_array_equal(o_ids.cpu().numpy(), rid)


def test_device_entry_point(ctx, oracle):
    import torch

    rng = np.random.default_rng(6)
    c = synth.mixture_centres(rng, 768, 128)
    db = synth.gaussian_mixture(rng, 12000, 768, centre_vectors=c)
    q = synth.gaussian_mixture(rng, 257, 768, centre_vectors=c)
    d_db = torch.from_numpy(db).cuda()
    d_q = torch.from_numpy(q).cuda()
    st = torch.cuda.current_stream().cuda_stream
    lat = slx.EmbeddingLattice.from_device(d_db.data_ptr(), 12000, 768, stream=st, ctx=ctx)
    d_ids = torch.empty((257, 10), dtype=torch.int64, device="cuda")
    d_dist = torch.empty((257, 10), dtype=torch.int64, device="cuda")
    lat.query_device(d_q.data_ptr(), 257, 10, d_ids.data_ptr(), d_dist.data_ptr(), stream=st)
    torch.cuda.synchronize()
    rid, rdist = _ref(oracle, db, q, 10)
    np.testing.assert_array_equal(d_dist.cpu().numpy().view(np.uint64), rdist)
    np.testing.assert_array_equal(d_ids.cpu().numpy(), rid)
