"""Writes the full-size golden fixtures of the benchmark configurations from the oracle.

The oracle (the C++ restatement of the reference's integer path) is too slow to run inside the GPU
test session at these sizes (the 18-layer Gemma prefill alone is minutes on a few host cores), so
its outputs for the seeded models and ids are computed here once and committed:

* encoder_q8_0_b4_t128.npz  -- the CPU-runnable encoder configuration (nomic-bert 12L d768, Q8_0):
  pooled Q30 int64 of 4 sequences of 128 ids (IntegerTransformerSource.Forward).
* encoder_q4_0_b2_t512.npz  -- the batched-encoder configuration (same architecture, Q4_0): pooled
  Q30 int64 of 2 sequences of 512 ids.
* gemma_q4_0_t512_greedy2.npz -- the Gemma-2B-shaped causal LM (18L d2048, Q4_0 + F16 norms): the
  last position's hidden state after the output norm for the 512-token prompt
  (IntegerCausalSource.ForwardCausal) and the first 2 greedy tokens of Generate.

Each fixture stores the SHA-256 of the GGUF file it was computed on, so a change in the model
generator shows up as a hash mismatch rather than as a parity failure.

    python tests/golden/make_golden.py [encoder_q8_0|encoder_q4_0|gemma ...]
"""
from __future__ import annotations

import hashlib
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from spatialdb_b200 import synth  # noqa: E402

ENC_VOCAB = synth.EncoderShape().vocab


def sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 24), b""):
            h.update(chunk)
    return h.hexdigest()


def encoder_ids(batch: int, seq: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, ENC_VOCAB, (batch, seq)).astype(np.int32)


CASES = {
    # name: (model function, batch, seq, ids seed)
    "encoder_q8_0": (synth.encoder_q8_0_model, 4, 128, 0),
    "encoder_q4_0": (synth.encoder_q4_0_model, 2, 512, 1),
}
FILES = {"encoder_q8_0": "encoder_q8_0_b4_t128.npz", "encoder_q4_0": "encoder_q4_0_b2_t512.npz",
         "gemma": "gemma_q4_0_t512_greedy2.npz"}


def make_encoder(name: str) -> None:
    import oracle

    model, B, T, seed = CASES[name]
    path = model()
    ids = encoder_ids(B, T, seed)
    t0 = time.time()
    pooled = oracle.Encoder(path).forward(ids)
    print(f"{name}: oracle {B}x{T} in {time.time() - t0:.1f} s", flush=True)
    np.savez_compressed(os.path.join(HERE, FILES[name]), ids=ids, pooled=pooled, gguf_sha256=sha256(path))


def make_gemma() -> None:
    import oracle

    path = synth.gemma_model()
    prompt = synth.gemma_prompts(1)[0]
    c = oracle.Causal(path)
    t0 = time.time()
    last = c.forward_last(prompt)
    print(f"gemma: forward_last T=512 in {time.time() - t0:.1f} s", flush=True)
    t0 = time.time()
    tokens = c.generate(prompt, 2)
    print(f"gemma: 2 greedy tokens in {time.time() - t0:.1f} s: {tokens.tolist()}", flush=True)
    np.savez_compressed(os.path.join(HERE, FILES["gemma"]), prompt=prompt, last=last, tokens=tokens,
                        gguf_sha256=sha256(path))


def main(names: list[str]) -> None:
    import oracle

    oracle.build()
    oracle.set_threads(os.cpu_count() or 1)
    for n in names or ["encoder_q8_0", "encoder_q4_0", "gemma"]:
        make_gemma() if n == "gemma" else make_encoder(n)


if __name__ == "__main__":
    main(sys.argv[1:])
