"""The committed full-size fixtures are the oracle's outputs (CPU; pins tests/golden/ to the oracle).

The GPU tests compare the library with these fixtures at the benchmark configurations' full sizes.
Here one sequence of the CPU-runnable encoder configuration (nomic-bert 12L d768, Q8_0, 128 ids) is
recomputed by the oracle and must equal the fixture, and every fixture's metadata is checked.
The Gemma and 512-token fixtures take minutes of oracle time and are regenerated only by
tests/golden/make_golden.py.
"""
import os

import numpy as np

from spatialdb_b200 import synth

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_fixture_metadata():
    e8 = np.load(os.path.join(GOLDEN, "encoder_q8_0_b4_t128.npz"))
    assert e8["ids"].shape == (4, 128) and e8["pooled"].shape == (4, 768) and e8["pooled"].dtype == np.int64
    e4 = np.load(os.path.join(GOLDEN, "encoder_q4_0_b2_t512.npz"))
    assert e4["ids"].shape == (2, 512) and e4["pooled"].shape == (2, 768)
    g = np.load(os.path.join(GOLDEN, "gemma_q4_0_t512_greedy2.npz"))
    assert g["prompt"].shape == (512,) and g["last"].shape == (2048,) and g["tokens"].shape == (2,)
    assert np.array_equal(g["prompt"], synth.gemma_prompts(1)[0])
    for f in (e8, e4, g):
        assert len(str(f["gguf_sha256"])) == 64


def test_encoder_fixture_is_the_oracle_output(oracle):
    import hashlib

    e8 = np.load(os.path.join(GOLDEN, "encoder_q8_0_b4_t128.npz"))
    path = synth.encoder_q8_0_model()
    h = hashlib.sha256(open(path, "rb").read()).hexdigest()
    assert h == str(e8["gguf_sha256"]), "the seeded model generator no longer writes the fixture's model"
    oracle.set_threads(os.cpu_count() or 1)
    got = oracle.Encoder(path).forward(e8["ids"][:1])
    np.testing.assert_array_equal(got, e8["pooled"][:1])
