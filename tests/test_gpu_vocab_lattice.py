"""GPU parity of the VocabLattice lm-head (Generate(useLattice: true, latticeK), IntegerCausalSource.cs:86-108,
PredictNextToken :149-157, Lattice/VocabLattice.cs:15-76) against the oracle, through the C ABI.

Candidate lists must equal the oracle's exact k-nearest rows in (distance, row) order, and the chosen
token must be the oracle's. The second model's token table plants the hard cases: duplicated rows (every
distance and every score tied in pairs), all-zero rows, components whose quantized values overflow
int32 and whose squares wrap mod 2^64, and rows holding inf and NaN.
"""
import numpy as np
import pytest

import spatialdb_b200 as slx
from spatialdb_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    return slx.Context(0)


def _planted_rows(V: int, d: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    half = V // 2
    rows = (rng.standard_normal((half, d)) * 0.05).astype(np.float32)
    rows[:8] = 0.0                                            # quantize to the zero vector
    rows[8:12] *= 40.0                                        # components beyond int32 once quantized
    rows[12, :4] = [60000.0, -60000.0, 65504.0, -30000.0]     # squares wrap mod 2^64
    rows[13, 3] = np.inf
    rows[14, 5] = np.nan
    rows[15, :] = rows[16, :]                                 # a duplicate inside the first half
    dup = rng.permutation(half)
    return np.concatenate([rows, rows[dup]], axis=0)         # every row twice


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    d = tmp_path_factory.mktemp("vocab_models")
    cau = synth.write_causal(str(d / "cau.gguf"), synth.CausalShape(layers=2, embd=128, heads=4, kv_heads=1, head_dim=64,
                                                                     ff=256, vocab=1000), seed=13)
    V, dm = 512, 64
    planted = synth.write_causal(str(d / "planted.gguf"), synth.CausalShape(layers=1, embd=dm, heads=2, kv_heads=1,
                                                                            head_dim=32, ff=96, vocab=V), seed=21,
                                 token_rows=_planted_rows(V, dm, 5))
    # 5000 rows: three 2048-row selection slices, duplicates and zero rows spread across them
    Vw = 5000
    rng = np.random.default_rng(8)
    wide_rows = (rng.standard_normal((Vw, dm)) * 0.05).astype(np.float32)
    wide_rows[4500:] = wide_rows[rng.permutation(2200)[:500]]
    wide_rows[[5, 2047, 2048, 4095, 4096, 4999]] = 0.0
    wide = synth.write_causal(str(d / "wide.gguf"), synth.CausalShape(layers=1, embd=dm, heads=2, kv_heads=1,
                                                                      head_dim=32, ff=96, vocab=Vw), seed=23,
                              token_rows=wide_rows)
    # Q8_0 weights and a width that is not a multiple of 8 (blocks straddle token rows)
    q8odd = synth.write_causal(str(d / "q8odd.gguf"), synth.CausalShape(layers=1, embd=100, heads=2, kv_heads=1,
                                                                        head_dim=50, ff=64, vocab=700), synth.Q8_0,
                               seed=24)
    return {"cau": cau, "planted": planted, "wide": wide, "q8odd": q8odd}


def _oracle_table(oracle, path: str, vocab: int, d: int) -> np.ndarray:
    """TokenEmbeddingsFloat: (float)(Half) of the dequantized token rows."""
    g = oracle.Gguf(path)
    try:
        f = g.read_f32("token_embd.weight")
    finally:
        g.close()
    rows = min(vocab, f.size // d)
    return oracle.half_to_float(oracle.float_to_half(f[: rows * d])).reshape(rows, d)


def _check_query(oracle, m, table, hidden, k):
    got = m.vocab_lattice_query(hidden, k)
    if k <= 0:
        assert got.shape == (hidden.shape[0], 0)
        return
    ids, _ = oracle.knn_l2(oracle.quantize_dense(table), oracle.quantize_dense(hidden), k)
    np.testing.assert_array_equal(got.astype(np.int64), ids, err_msg=f"k={k}")


@pytest.mark.parametrize("name", ["cau", "planted", "wide", "q8odd"])
def test_query_topk_matches_oracle(ctx, oracle, models, name):
    path = models[name]
    m = slx.IntegerCausalSource.load(path, ctx=ctx)
    table = _oracle_table(oracle, path, m.vocab, m.embd)
    V, d = table.shape
    rng = np.random.default_rng(7)
    hidden = (rng.standard_normal((11, d)) * 3.0).astype(np.float32)   # quantized beyond int32
    hidden[1] *= 0.01
    hidden[2, rng.random(d) < 0.3] = 0.0005                              # below the zero threshold
    hidden[3] = 0.0                                                      # distances = row norms
    finite = np.flatnonzero(np.isfinite(table).all(axis=1))
    hidden[4] = table[finite[-1]]                                        # distance 0 to a row (and its twin)
    hidden[5] = table[finite[len(finite) // 2]] + 0.0004
    hidden[6] = hidden[4]                                                # duplicate queries
    hidden[7, :3] = [1e4, -2e4, 3e4]
    for k in (0, 1, 2, 7, 64, 255, 512, 513, V - 1, V, V + 9):
        _check_query(oracle, m, table, hidden, k)


def test_query_distances_cover_every_half(ctx, oracle, tmp_path):
    """A token table holding all 65536 Half bit patterns once (1024 rows x 64): with k = V the exact
    distance of every row is compared, which pins the device's quantization of every Half value."""
    V, dm = 1024, 64
    bits = np.random.default_rng(3).permutation(65536).astype(np.uint16)
    rows = bits.view(np.float16).astype(np.float32).reshape(V, dm)
    path = synth.write_causal(str(tmp_path / "halves.gguf"), synth.CausalShape(layers=1, embd=dm, heads=2, kv_heads=1,
                                                                              head_dim=32, ff=96, vocab=V), seed=22,
                              token_rows=rows)
    m = slx.IntegerCausalSource.load(path, ctx=ctx)
    table = _oracle_table(oracle, path, m.vocab, m.embd)
    hidden = (np.random.default_rng(9).standard_normal((5, dm)) * 2.0).astype(np.float32)
    hidden[0] = 0.0
    got_ids, got_dist = m.vocab_lattice_query(hidden, V, return_distances=True)
    ids, dist = oracle.knn_l2(oracle.quantize_dense(table), oracle.quantize_dense(hidden), V)
    np.testing.assert_array_equal(got_dist, dist)
    np.testing.assert_array_equal(got_ids.astype(np.int64), ids)


@pytest.mark.parametrize("name", ["cau", "planted", "wide", "q8odd"])
def test_lattice_next_token_matches_oracle(ctx, oracle, models, name):
    path = models[name]
    m = slx.IntegerCausalSource.load(path, ctx=ctx)
    o = oracle.Causal(path)
    rng = np.random.default_rng(61)
    lo = 20 if name == "planted" else 0  # prompts avoid the planted inf / NaN rows
    batch = rng.integers(lo, o.vocab // 2, (4, 9)).astype(np.int32)
    # the brute-force head on the same models, one and several queries per block
    expect = [o.next_token(batch[b]) for b in range(len(batch))]
    assert list(m.next_token(batch)) == expect
    assert list(m.next_token(batch[:1])) == expect[:1]
    wide_batch = rng.integers(lo, o.vocab // 2, (19, 5)).astype(np.int32)
    assert list(m.next_token(wide_batch)) == [o.next_token(wide_batch[b]) for b in range(len(wide_batch))]
    for k in (0, 1, 3, 64, 300, o.vocab, o.vocab + 5):
        nx = m.next_token(batch, use_lattice=True, lattice_k=k)
        assert list(nx) == [o.next_token_lattice(batch[b], k) for b in range(len(batch))], f"k={k}"


def test_lattice_generate_matches_oracle(ctx, oracle, models):
    path = models["cau"]
    m = slx.IntegerCausalSource.load(path, ctx=ctx)
    o = oracle.Causal(path)
    rng = np.random.default_rng(71)
    prompts = rng.integers(0, o.vocab, (2, 13)).astype(np.int32)
    for k in (8, 64):
        gen = m.generate(prompts, 6, use_lattice=True, lattice_k=k)
        for b in range(2):
            np.testing.assert_array_equal(gen[b], o.generate_lattice(prompts[b], 6, k), err_msg=f"k={k} b={b}")
    # the full-vocabulary lattice scores every row: the same tokens as the argmax head
    full = m.generate(prompts[:1], 4, use_lattice=True, lattice_k=o.vocab)[0]
    np.testing.assert_array_equal(full, m.generate(prompts[:1], 4)[0])


def test_lattice_k_limit(ctx, models):
    m = slx.IntegerCausalSource.load(models["cau"], ctx=ctx)
    with pytest.raises(slx.SlxError):
        m.next_token(np.zeros((1, 3), np.int32), use_lattice=True, lattice_k=8193)
