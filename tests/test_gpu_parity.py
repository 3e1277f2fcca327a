"""GPU parity: libslx (through its C ABI) against the oracle on the same seeded inputs.

Integer outputs must be bit-identical (the reference is exact Int128 arithmetic); the float L2
output is compared bit for bit too, since both sides run the same sequential fp32 loop.
"""
import os

import numpy as np
import pytest

import spatialdb_b200 as slx
from spatialdb_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    return slx.Context(0)


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    d = tmp_path_factory.mktemp("models")
    enc = synth.write_encoder(str(d / "enc.gguf"), synth.EncoderShape(layers=2, embd=64, heads=4, ff=160, vocab=777, ctx=512),
                              synth.Q8_0, seed=11)
    enc4 = synth.write_encoder(str(d / "enc4.gguf"), synth.EncoderShape(layers=2, embd=96, heads=3, ff=192, vocab=500, ctx=512),
                               synth.Q4_0, seed=12)
    cau = synth.write_causal(str(d / "cau.gguf"), synth.CausalShape(layers=2, embd=128, heads=4, kv_heads=1, head_dim=64,
                                                                     ff=256, vocab=1000), seed=13)
    cau_sw = synth.write_causal(str(d / "cau_sw.gguf"), synth.CausalShape(layers=7, embd=64, heads=2, kv_heads=1, head_dim=32,
                                                                          ff=96, vocab=300, sliding_window=5), seed=14,
                                qk_norm=False)
    # FFN activations beyond five digits: the gate/up and down projections take their exact kernels
    big = synth.write_encoder(str(d / "big.gguf"), synth.EncoderShape(layers=2, embd=64, heads=4, ff=128, vocab=300, ctx=512),
                              synth.Q8_0, seed=15, ffn_norm_scale=1000.0)
    # the first block's q and k beyond five digits: the attention's exact fallback (q and k rotated first)
    bigq = synth.write_encoder(str(d / "bigq.gguf"), synth.EncoderShape(layers=2, embd=64, heads=4, ff=128, vocab=300,
                                                                        ctx=512), synth.Q8_0, seed=16, embd_norm_scale=3000.0)
    return {"enc": enc, "enc4": enc4, "cau": cau, "cau_sw": cau_sw, "big": big, "bigq": bigq}


# ------------------------------------------------------------------ dequant
@pytest.mark.parametrize("dtype", [synth.F32, synth.F16, synth.BF16, synth.Q8_0, synth.Q4_0, synth.Q2_K, synth.Q3_K,
                                   synth.Q4_K, synth.Q5_K, synth.Q6_K, synth.Q8_K])
def test_dequantize_matches_oracle(ctx, oracle, dtype):
    rng = np.random.default_rng(dtype)
    n = 256 * 37
    nbytes = synth.block_bytes(dtype, n)
    raw = rng.integers(0, 256, nbytes, dtype=np.uint16).astype(np.uint8)
    if dtype in (synth.F16, synth.BF16):  # keep the payload finite-ish but include specials
        raw[:8] = [0x00, 0x7C, 0x00, 0xFC, 0x01, 0x7C, 0x00, 0x80]
    if dtype == synth.Q8_K:  # f32 scales at the start of each super-block: make them finite
        for sb in range(n // 256):
            raw[sb * 292: sb * 292 + 4] = np.frombuffer(np.float32(rng.standard_normal()).tobytes(), np.uint8)
    got = slx.dequantize(dtype, raw, n, ctx)
    ref = oracle.dequantize(dtype, raw, n)
    np.testing.assert_array_equal(got.view(np.uint32)[~np.isnan(ref)], ref.view(np.uint32)[~np.isnan(ref)])
    assert np.isnan(got[np.isnan(ref)]).all()


def test_dequantize_mxfp4(ctx, oracle):
    rng = np.random.default_rng(3)
    blocks = rng.integers(0, 15, (64, 32)).astype(np.uint8)
    raw = np.concatenate([rng.integers(100, 140, (64, 1)).astype(np.uint8), blocks[:, 0::2] | (blocks[:, 1::2] << 4)], 1).reshape(-1)
    np.testing.assert_array_equal(slx.dequantize(synth.MXFP4, raw, 64 * 32, ctx), oracle.dequantize(synth.MXFP4, raw, 64 * 32))
    raw[5] = 0xF0
    with pytest.raises(slx.IndexOutOfRangeError):
        slx.dequantize(synth.MXFP4, raw, 64 * 32, ctx)


# ------------------------------------------------------------------ matmul
def _q30_weight(oracle, dtype, raw, n, half):
    f = oracle.dequantize(dtype, raw, n)
    if half:
        return oracle.float_to_half(f)
    return oracle.quantize_from_float(f)


@pytest.mark.parametrize("dtype,half", [(synth.Q8_0, False), (synth.Q4_0, False), (synth.Q8_0, True), (synth.Q4_0, True),
                                        (synth.F16, False), (synth.F32, True)])
@pytest.mark.parametrize("M,K,N", [(1, 64, 40), (37, 96, 130), (130, 160, 70)])
def test_matmul_q30_matches_oracle(ctx, oracle, dtype, half, M, K, N):
    rng = np.random.default_rng(M * 1000 + K + N + dtype)
    if dtype == synth.Q8_0:
        raw = synth.random_q8_0(rng, N * K)
    elif dtype == synth.Q4_0:
        raw = synth.random_q4_0(rng, N * K)
    else:
        raw = synth.encode(dtype, rng.standard_normal(N * K).astype(np.float32) * 0.05)
    a = rng.integers(-(1 << 40), 1 << 40, (M, K), dtype=np.int64)
    a[0, : min(K, 4)] = [np.iinfo(np.int64).max, np.iinfo(np.int64).min, -1, 1][: min(K, 4)]
    got = slx.matmul_q30(a, dtype, raw, N, half_composite=half, shift=30, ctx=ctx)
    w = _q30_weight(oracle, dtype, raw, N * K, half)
    ref = (oracle.matmul_half(a, M, K, w, N, 30, 30) if half else oracle.matmul_long(a, M, K, w, N, 30)).reshape(M, N)
    np.testing.assert_array_equal(got, ref)


def test_matmul_shift_zero_and_unaligned_k(ctx, oracle):
    rng = np.random.default_rng(5)
    M, K, N = 9, 48, 33  # K not a multiple of 32: blocks straddle rows in flat order
    raw = synth.random_q8_0(rng, N * K)
    a = rng.integers(-(1 << 20), 1 << 20, (M, K), dtype=np.int64)
    for shift in (0, 7, 30):
        got = slx.matmul_q30(a, synth.Q8_0, raw, N, shift=shift, ctx=ctx)
        w = oracle.quantize_from_float(oracle.dequantize(synth.Q8_0, raw, N * K))
        np.testing.assert_array_equal(got, oracle.matmul_long(a, M, K, w, N, shift).reshape(M, N))


# ------------------------------------------------------------------ encoder
@pytest.mark.parametrize("name", ["enc", "enc4"])
def test_encoder_layers_and_pool(ctx, oracle, models, name):
    path = models[name]
    m = slx.IntegerTransformerSource.load(path, ctx=ctx)
    o = oracle.Encoder(path)
    rng = np.random.default_rng(21)
    ids = rng.integers(0, o.vocab, 33).astype(np.int32)
    ids[3] = -5            # negative id -> UNK row
    ids[7] = o.vocab + 10  # past the table -> UNK row
    for nl in range(o.layers + 1):
        np.testing.assert_array_equal(m.trace_hidden(ids, nl), o.hidden(ids, nl), err_msg=f"layer {nl}")
    B = 3
    batch = rng.integers(0, o.vocab, (B, 40)).astype(np.int32)
    np.testing.assert_array_equal(m.forward(batch), o.forward(batch))
    l2 = m.forward_float(batch)
    for b in range(B):
        ref = oracle.to_float_l2(o.forward(batch[b:b + 1])[0])
        np.testing.assert_array_equal(l2[b].view(np.uint32), ref.view(np.uint32))


def test_encoder_ffn_beyond_digit_range(ctx, oracle, models):
    """The FFN's activations exceed the five-digit range: the gate/up projections and the down
    projection (reading the SiLU gate's planes) fall back to their exact kernels."""
    path = models["big"]
    m = slx.IntegerTransformerSource.load(path, ctx=ctx)
    o = oracle.Encoder(path)
    batch = np.random.default_rng(5).integers(0, o.vocab, (2, 24)).astype(np.int32)
    for nl in range(o.layers + 1):
        np.testing.assert_array_equal(m.trace_hidden(batch[0], nl), o.hidden(batch[0], nl), err_msg=f"layer {nl}")
    np.testing.assert_array_equal(m.forward(batch), o.forward(batch))


def test_encoder_attention_beyond_digit_range(ctx, oracle, models):
    """q and k of the first block exceed the five-digit range after RoPE: the attention's exact kernel
    runs on q and k that are rotated in place first (the fast path rotates only their digit planes)."""
    path = models["bigq"]
    m = slx.IntegerTransformerSource.load(path, ctx=ctx)
    o = oracle.Encoder(path)
    batch = np.random.default_rng(6).integers(0, o.vocab, (2, 20)).astype(np.int32)
    for nl in range(o.layers + 1):
        np.testing.assert_array_equal(m.trace_hidden(batch[0], nl), o.hidden(batch[0], nl), err_msg=f"layer {nl}")
    np.testing.assert_array_equal(m.forward(batch), o.forward(batch))


def test_encoder_graph_replay_across_shapes(ctx, oracle, models):
    """Repeated calls of one shape replay the forward from the library's CUDA graph (captured on the
    second call); a larger shape reallocates the workspaces, after which the first shape runs eagerly
    and is captured again. Every call equals the oracle."""
    m = slx.IntegerTransformerSource.load(models["enc"], ctx=ctx)
    o = oracle.Encoder(models["enc"])
    rng = np.random.default_rng(9)
    for B, T in [(2, 40)] * 4 + [(4, 64)] * 2 + [(2, 40)] * 3:
        batch = rng.integers(0, o.vocab, (B, T)).astype(np.int32)
        np.testing.assert_array_equal(m.forward(batch), o.forward(batch), err_msg=f"{B} x {T}")


def test_encoder_edge_shapes(ctx, oracle, models):
    m = slx.IntegerTransformerSource.load(models["enc"], ctx=ctx)
    o = oracle.Encoder(models["enc"])
    one = np.array([[5]], np.int32)
    np.testing.assert_array_equal(m.forward(one), o.forward(one))
    empty = np.zeros((2, 0), np.int32)
    np.testing.assert_array_equal(m.forward(empty), np.zeros((2, m.embd), np.int64))
    long = np.random.default_rng(1).integers(0, o.vocab, (1, 512)).astype(np.int32)
    np.testing.assert_array_equal(m.forward(long), o.forward(long))
    with pytest.raises(slx.IndexOutOfRangeError):  # RoPE table has 512 rows
        m.forward(np.zeros((1, 513), np.int32))


# ------------------------------------------------------------------ causal
def test_causal_forward_and_generate(ctx, oracle, models):
    path = models["cau"]
    m = slx.IntegerCausalSource.load(path, ctx=ctx)
    o = oracle.Causal(path)
    rng = np.random.default_rng(31)
    ids = rng.integers(0, o.vocab, 19).astype(np.int32)
    for nl in range(o.layers + 1):
        np.testing.assert_array_equal(m.trace_hidden(ids, nl), o.hidden(ids, nl), err_msg=f"layer {nl}")
    np.testing.assert_array_equal(m.forward_causal(ids), o.forward_last(ids))
    assert m.next_token(ids)[0] == o.next_token(ids)
    gen = m.generate(ids[None], 6)[0]
    np.testing.assert_array_equal(gen, o.generate(ids, 6))
    batch = rng.integers(0, o.vocab, (3, 11)).astype(np.int32)
    nx = m.next_token(batch)
    assert list(nx) == [o.next_token(batch[b]) for b in range(3)]


def test_causal_sliding_window_and_missing_norms(ctx, oracle, models):
    path = models["cau_sw"]  # 7 layers: layer 5 is global, the rest sliding (window 5); no q/k norms
    m = slx.IntegerCausalSource.load(path, ctx=ctx)
    o = oracle.Causal(path)
    ids = np.random.default_rng(41).integers(0, o.vocab, 14).astype(np.int32)
    for nl in range(o.layers + 1):
        np.testing.assert_array_equal(m.trace_hidden(ids, nl), o.hidden(ids, nl), err_msg=f"layer {nl}")
    np.testing.assert_array_equal(m.generate(ids[None], 4)[0], o.generate(ids, 4))


def test_gemma_encoder(ctx, oracle, models):
    path = models["cau"]
    m = slx.IntegerGemmaSource.load(path, ctx=ctx)
    o = oracle.Causal(path, gemma_encoder=True)
    batch = np.random.default_rng(51).integers(0, o.vocab, (2, 13)).astype(np.int32)
    np.testing.assert_array_equal(m.forward(batch), o.encode_pooled(batch))


# ------------------------------------------------------------------ errors
def test_load_errors(ctx, tmp_path, models):
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"\0\0\0\0\2\0\0\0")
    with pytest.raises(slx.InvalidDataError):
        slx.IntegerTransformerSource.load(str(bad), ctx=ctx)
    with pytest.raises(slx.NotFoundError):
        slx.IntegerTransformerSource.load(str(tmp_path / "missing.gguf"), ctx=ctx)
    with pytest.raises(slx.NotSupportedError):
        slx.IntegerTransformerSource.load(models["cau"], ctx=ctx)
    with pytest.raises(slx.NotSupportedError):
        slx.IntegerCausalSource.load(models["enc"], ctx=ctx)
