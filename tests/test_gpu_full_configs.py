"""Bit-exact parity at the benchmark configurations' full sizes, against the oracle's outputs.

The oracle is too slow to run at these sizes inside the test session (the 18-layer Gemma prefill
takes minutes on the host cores), so its outputs were computed once by tests/golden/make_golden.py
and committed as fixtures; each fixture carries the SHA-256 of the seeded GGUF model it was
computed on, which is checked first. Models and ids are regenerated here from their seeds.

* CPU-runnable encoder configuration: nomic-bert 12L d768 H12 F3072 V30522, Q8_0, 4 x 128 ids,
  pooled Q30 int64 (IntegerTransformerSource.Forward, Gguf/IntegerTransformerSource.cs:65-78).
* Batched-encoder configuration: the same architecture with Q4_0 weights, 2 x 512 ids.
* Gemma-2B-shaped causal LM: 18L d2048 8q/1kv hd256 F16384 V256000, Q4_0 + F16 norms, a 512-token
  prompt: the last hidden state after the output norm (ForwardCausal,
  Gguf/IntegerCausalSource.cs:128-147) and the first two greedy tokens of Generate (:86-108).
"""
import hashlib
import os

import numpy as np
import pytest

import spatialdb_b200 as slx
from spatialdb_b200 import synth

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _fixture(name: str, model_path: str) -> dict:
    f = dict(np.load(os.path.join(GOLDEN, name)))
    h = hashlib.sha256()
    with open(model_path, "rb") as fh:
        for chunk in iter(lambda: fh.read(1 << 24), b""):
            h.update(chunk)
    assert h.hexdigest() == str(f["gguf_sha256"]), f"{model_path}: not the model {name} was computed on"
    return f


@pytest.fixture(scope="module")
def ctx():
    return slx.Context(0)


@pytest.mark.parametrize("name,model", [("encoder_q8_0_b4_t128.npz", synth.encoder_q8_0_model),
                                        ("encoder_q4_0_b2_t512.npz", synth.encoder_q4_0_model)])
def test_encoder_configuration_matches_oracle(ctx, name, model):
    path = model()
    g = _fixture(name, path)
    m = slx.IntegerTransformerSource.load(path, ctx=ctx)
    got = m.forward(g["ids"])
    np.testing.assert_array_equal(got, g["pooled"])
    # the same batch through the device entry point
    import torch

    stream = torch.cuda.Stream()
    d_ids = torch.from_numpy(g["ids"]).cuda()
    pooled = torch.empty(g["pooled"].shape, dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()
    m.encode_device(d_ids.data_ptr(), *g["ids"].shape, pooled.data_ptr(), stream.cuda_stream)
    ctx.status(stream.cuda_stream)
    np.testing.assert_array_equal(pooled.cpu().numpy(), g["pooled"])
    m.close()


def test_gemma_configuration_matches_oracle(ctx):
    path = synth.gemma_model()
    g = _fixture("gemma_q4_0_t512_greedy2.npz", path)
    assert np.array_equal(g["prompt"], synth.gemma_prompts(1)[0])
    m = slx.IntegerCausalSource.load(path, ctx=ctx)
    np.testing.assert_array_equal(m.forward_causal(g["prompt"]), g["last"])
    toks = m.generate(g["prompt"][None], 2)[0]
    np.testing.assert_array_equal(toks, g["tokens"])
    m.close()
