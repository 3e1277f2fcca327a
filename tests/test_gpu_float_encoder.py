"""GPU parity of the fp32 encoder twin (TransformerEmbeddingSource, Gguf/TransformerEmbeddingSource.cs)
against the oracle's restatement, through the C ABI.

The reference's dot products are Vector<float> SIMD sums (lane order machine-dependent), so the bar
is a tolerance on the L2-normalised outputs: maximum absolute error <= 1e-4 and cosine >= 0.9999
per sequence."""
import numpy as np
import pytest

import spatialdb_b200 as slx
from spatialdb_b200 import synth

pytestmark = pytest.mark.gpu

MAX_ABS = 1e-4
MIN_COS = 0.9999


@pytest.fixture(scope="module")
def ctx():
    return slx.Context(0)


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    d = tmp_path_factory.mktemp("float_models")
    return {
        "q8": synth.write_encoder(str(d / "q8.gguf"), synth.EncoderShape(layers=2, embd=64, heads=4, ff=160, vocab=777,
                                                                         ctx=512), synth.Q8_0, seed=11),
        "q4": synth.write_encoder(str(d / "q4.gguf"), synth.EncoderShape(layers=2, embd=96, heads=3, ff=192, vocab=500,
                                                                         ctx=512), synth.Q4_0, seed=12),
        "wide": synth.write_encoder(str(d / "wide.gguf"), synth.EncoderShape(layers=3, embd=768, heads=12, ff=3072,
                                                                             vocab=3000, ctx=512), synth.Q8_0, seed=13),
        # the CPU-runnable reference configuration's architecture: 12 layers, d 768, FFN 3072, vocab 30522
        "full": synth.write_encoder(str(d / "full.gguf"), synth.EncoderShape(layers=12, embd=768, heads=12, ff=3072,
                                                                             vocab=30522, ctx=512), synth.Q8_0, seed=0),
    }


def _check(got, want):
    got = np.atleast_2d(got)
    want = np.atleast_2d(want)
    assert got.shape == want.shape
    err = float(np.abs(got - want).max())
    cos = (got * want).sum(1) / (np.linalg.norm(got, axis=1) * np.linalg.norm(want, axis=1))
    assert err <= MAX_ABS, f"max abs error {err}"
    assert cos.min() >= MIN_COS, f"cosine {cos.min()}"


@pytest.mark.parametrize("name,T,B", [("q8", 1, 2), ("q8", 37, 3), ("q8", 512, 1), ("q4", 64, 2), ("wide", 48, 2),
                                      ("full", 128, 2)])
def test_float_encoder_matches_oracle(ctx, oracle, models, name, T, B):
    m = slx.TransformerEmbeddingSource.load(models[name], ctx=ctx)
    o = oracle.FloatEncoder(models[name])
    rng = np.random.default_rng(T * 7 + B)
    ids = rng.integers(0, m.vocab, (B, T)).astype(np.int32)
    got = m.forward(ids)
    want = np.stack([o.forward(ids[b]) for b in range(B)])
    _check(got, want)
    np.testing.assert_allclose(np.linalg.norm(got, axis=1), 1.0, atol=1e-5)


def test_float_encoder_unk_ids_and_limits(ctx, oracle, models):
    m = slx.TransformerEmbeddingSource.load(models["q8"], ctx=ctx)
    o = oracle.FloatEncoder(models["q8"])
    ids = np.array([[-5, 3, 10 ** 6, 7, 776, 777]], np.int32)  # out-of-range ids take the UNK row
    _check(m.forward(ids), o.forward(ids[0])[None])
    with pytest.raises(slx.IndexOutOfRangeError):
        m.forward(np.zeros((1, 513), np.int32))  # the 512-row RoPE cache
    with pytest.raises(slx.SlxError):
        m.trace_hidden(np.zeros(4, np.int32))  # no Q30 trace on the float twin


def test_float_encoder_close_to_integer_encoder(ctx, models):
    """Both encoders compute the same function (the integer one exactly in Q30): their L2-normalised
    outputs agree to the integer path's fixed-point rounding."""
    f = slx.TransformerEmbeddingSource.load(models["q8"], ctx=ctx)
    q = slx.IntegerTransformerSource.load(models["q8"], ctx=ctx)
    ids = np.random.default_rng(3).integers(0, f.vocab, (2, 40)).astype(np.int32)
    a = f.forward(ids)
    b = q.forward_float(ids)
    cos = (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))
    assert cos.min() >= 0.999
