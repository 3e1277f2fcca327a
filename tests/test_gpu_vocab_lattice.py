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
    return {"cau": cau, "planted": planted}


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


@pytest.mark.parametrize("name", ["cau", "planted"])
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
    for k in (0, 1, 2, 7, 64, 255, V - 1, V, V + 9):
        _check_query(oracle, m, table, hidden, k)


@pytest.mark.parametrize("name", ["cau", "planted"])
def test_lattice_next_token_matches_oracle(ctx, oracle, models, name):
    path = models[name]
    m = slx.IntegerCausalSource.load(path, ctx=ctx)
    o = oracle.Causal(path)
    rng = np.random.default_rng(61)
    lo = 20 if name == "planted" else 0  # prompts avoid the planted inf / NaN rows
    batch = rng.integers(lo, o.vocab // 2, (4, 9)).astype(np.int32)
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
