"""Gemma-2B-shaped causal LM at full width (d 2048, 8 query / 1 KV head of 256, FFN 16384, vocab
256000, Q4_0 projections and embeddings, F16 norms) with 2 of its 18 layers: hidden states, the last
position, greedy next tokens and a short generation, bit-exact against the oracle. This is the
reduced-depth parity check of the causal benchmark configuration."""
import numpy as np
import pytest

import spatialdb_b200 as slx
from spatialdb_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model_path(tmp_path_factory):
    shape = synth.CausalShape(layers=2)
    return synth.write_causal(str(tmp_path_factory.mktemp("gemma") / "g2.gguf"), shape, synth.Q4_0, synth.F16, seed=5,
                              eos=shape.vocab - 1)


def test_gemma_width_parity(model_path, oracle):
    ctx = slx.Context(0)
    m = slx.IntegerCausalSource.load(model_path, ctx=ctx)
    o = oracle.Causal(model_path)
    assert (m.embd, m.heads, m.kv_heads, m.head_dim, m.ff, m.vocab) == (2048, 8, 1, 256, 16384, 256000)
    ids = np.random.default_rng(3).integers(0, 255999, 64).astype(np.int32)
    np.testing.assert_array_equal(m.trace_hidden(ids, 1), o.hidden(ids, 1))
    np.testing.assert_array_equal(m.forward_causal(ids), o.forward_last(ids))
    assert int(m.next_token(ids[None])[0]) == o.next_token(ids)
    np.testing.assert_array_equal(m.generate(ids[None], 3)[0], o.generate(ids, 3))
