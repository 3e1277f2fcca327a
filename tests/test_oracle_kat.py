"""The oracle against the reference's own known-answer tests.

Each test ports one of SparseLattice.Test's unit tests (file:line cited) and runs it on the oracle,
so the oracle is pinned by the same answers that pin the C# reference. Random inputs in the C#
tests come from System.Random; here they come from a seeded numpy generator with the same ranges,
which is all those property-style tests depend on.
"""
import math
import os
import struct

import numpy as np
import pytest

from spatialdb_b200 import synth

FRAC = 30
ONE = 1 << 30
MAXL = (1 << 63) - 1


def fixed_from_double(v, frac=FRAC):
    return int(v * (1 << frac))


def to_double(v, frac=FRAC):
    return v / float(1 << frac)


def _raw_gguf(path, version=3, meta=(("general.architecture", synth.T_STRING, "bert"),), tensor=None):
    """WriteTempGguf / WriteRawTensorGguf (GgufReaderTests.cs:19-100, 514-545)."""
    w = synth.GgufWriter(version)
    for k, t, v in meta:
        w.kv(k, t, v)
    if tensor is not None:
        name, shape, dtype, raw = tensor
        w.tensor_raw(name, shape, dtype, np.frombuffer(bytes(raw), np.uint8))
    return w.write(str(path))


# ---------------------------------------------------------------- GgufReaderTests.cs
def test_open_bad_magic(oracle, tmp_path):  # GgufReaderTests.cs:103-115
    p = tmp_path / "bad.gguf"
    p.write_bytes(bytes([0, 0, 0, 0, 2, 0, 0, 0]))
    with pytest.raises(oracle.OracleError) as e:
        oracle.Gguf(str(p))
    assert e.value.status == 2


def test_open_unsupported_version(oracle, tmp_path):  # GgufReaderTests.cs:117-133
    p = tmp_path / "v1.gguf"
    p.write_bytes(struct.pack("<IIQQ", 0x46554747, 1, 0, 0))
    with pytest.raises(oracle.OracleError) as e:
        oracle.Gguf(str(p))
    assert e.value.status == 2


def test_open_missing_file(oracle, tmp_path):  # GgufReaderTests.cs:135-140
    with pytest.raises(oracle.OracleError) as e:
        oracle.Gguf(str(tmp_path / "does_not_exist.gguf"))
    assert e.value.status == 3


def test_metadata_roundtrip(oracle, tmp_path):  # GgufReaderTests.cs:146-198
    p = _raw_gguf(tmp_path / "m.gguf", meta=[
        ("general.architecture", synth.T_STRING, "bert"),
        ("bert.embedding_length", synth.T_UINT32, 768),
        ("bert.context_length", synth.T_UINT32, 512),
        ("bert.attention.head_count", synth.T_UINT32, 12),
        ("bert.block_count", synth.T_UINT32, 6),
        ("bert.feed_forward_length", synth.T_UINT32, 3072),
    ])
    info = oracle.Gguf(p).info()
    assert info["version"] == 3 and info["arch"] == "bert"
    assert (info["embd"], info["ctx"], info["heads"], info["layers"], info["ff"]) == (768, 512, 12, 6, 3072)
    p2 = _raw_gguf(tmp_path / "m2.gguf")
    info2 = oracle.Gguf(p2).info()
    assert (info2["embd"], info2["heads"], info2["layers"]) == (0, 0, 0)


def test_f32_tensor_roundtrip(oracle, tmp_path):  # GgufReaderTests.cs:206-224, 226-236
    orig = np.array([1.0, -2.0, 3.14, 0.0, -0.001], np.float32)
    p = _raw_gguf(tmp_path / "f.gguf", tensor=("test_tensor", (5,), synth.F32, orig.tobytes()))
    g = oracle.Gguf(p)
    np.testing.assert_array_equal(g.read_f32("test_tensor"), orig)
    with pytest.raises(oracle.OracleError) as e:
        g.read_f32("does_not_exist")
    assert e.value.status == 3


def test_half_to_float_known_values(oracle):  # GgufReaderTests.cs:243-264
    cases = {0x3C00: 1.0, 0xBC00: -1.0, 0x0000: 0.0, 0x3800: 0.5, 0xB800: -0.5, 0x4000: 2.0}
    for h, f in cases.items():
        assert oracle.half_to_float(np.array([h], np.uint16))[0] == f


def test_half_conversions_match_ieee(oracle):
    """HalfToFloat is exact and (Half)float is round-to-nearest-even: both equal numpy's IEEE casts."""
    allh = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    got = oracle.half_to_float(allh)
    ref = allh.view(np.float16).astype(np.float32)
    nan = np.isnan(ref)
    np.testing.assert_array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32))
    assert np.isnan(got[nan]).all()
    rng = np.random.default_rng(1)
    bits = rng.integers(0, 1 << 32, size=2_000_000, dtype=np.uint64).astype(np.uint32)
    edge = np.array([0x477FEFFF, 0x477FF000, 0x477FF001, 0x33000000, 0x33000001, 0x387FE000, 0x387FF000,
                     0x38800000, 0x3F800000, 0x7F800000, 0xFF800000, 0x00000001, 0x80000000], np.uint32)
    f = np.concatenate([bits, edge]).view(np.float32)
    got = oracle.float_to_half(f)
    with np.errstate(over="ignore"):
        ref = f.astype(np.float16).view(np.uint16)
    finite = ~np.isnan(f)
    np.testing.assert_array_equal(got[finite], ref[finite])


def test_q8_0_single_block(oracle, tmp_path):  # GgufReaderTests.cs:266-297
    block = bytes([0x00, 0x38]) + bytes((i - 16) & 0xFF for i in range(32))
    p = _raw_gguf(tmp_path / "q8.gguf", tensor=("q8_tensor", (32,), synth.Q8_0, block))
    out = oracle.Gguf(p).read_f32("q8_tensor")
    np.testing.assert_array_equal(out, 0.5 * (np.arange(32) - 16).astype(np.float32))


def test_q4_0_single_block_interleave(oracle, tmp_path):  # GgufReaderTests.cs:299-338
    raw = bytearray([0x00, 0x3C])
    for j in range(16):
        lo, hi = (2 * j) % 16, (2 * j + 1) % 16
        raw.append((hi << 4) | lo)
    p = _raw_gguf(tmp_path / "q4.gguf", tensor=("q4_tensor", (32,), synth.Q4_0, bytes(raw)))
    out = oracle.Gguf(p).read_f32("q4_tensor")
    exp = []
    for i in range(32):
        b = raw[2 + i // 2]
        nib = (b & 0x0F) if i % 2 == 0 else (b >> 4)
        exp.append(float(nib - 8))
    np.testing.assert_array_equal(out, np.array(exp, np.float32))


def test_has_tensor_and_table(oracle, tmp_path):  # GgufReaderTests.cs:340-370
    p = _raw_gguf(tmp_path / "t.gguf", tensor=("token_embd.weight", (2,), synth.F32, np.array([1, 2], np.float32).tobytes()))
    g = oracle.Gguf(p)
    assert g.elements("token_embd.weight") == 2 and g.elements("no_such_tensor") == -1
    assert g.info()["n_tensors"] == 1


def test_truncated_tensor_is_eof(oracle, tmp_path):  # GgufDequantizer.ReadExact (GgufDequantizer.cs:330-343)
    block = bytes([0x00, 0x38]) + bytes(32)
    p = _raw_gguf(tmp_path / "q8t.gguf", tensor=("q8", (32,), synth.Q8_0, block))
    data = open(p, "rb").read()
    open(p, "wb").write(data[:-5])
    with pytest.raises(oracle.OracleError) as e:
        oracle.Gguf(p).read_f32("q8")
    assert e.value.status == 5


def test_mxfp4_table_quirk(oracle):
    """GgufDequantizer.cs:91-95: the missing comma folds -4 and -6 into -10; nibble 15 is out of range."""
    blk = bytes([127]) + bytes([(14 << 4) | 7] + [0x10] * 15)
    out = oracle.dequantize(synth.MXFP4, blk, 32)
    assert out[0] == 6.0 and out[1] == -10.0 and out[2] == 0.0 and out[3] == 0.5
    with pytest.raises(oracle.OracleError) as e:
        oracle.dequantize(synth.MXFP4, bytes([127]) + bytes([0xF0] + [0] * 15), 32)
    assert e.value.status == 6


def test_kquant_decoders_follow_reference_element_order(oracle):
    """K-quant orders as written in GgufDequantizer.cs:125-324 (not pinned by the reference's tests)."""
    rng = np.random.default_rng(3)
    # Q4_K with d=1, dmin=0: element j is nibble (j%2 ? hi : lo) of byte j/2, times its sub-block scale
    raw = bytearray(144)
    raw[0:2] = np.float16(1.0).tobytes()
    raw[2:4] = np.float16(0.0).tobytes()
    sc = bytes([1, 2, 3, 4, 0, 0, 0, 0, 5, 6, 7, 8])
    raw[4:16] = sc
    qs = rng.integers(0, 256, 128, dtype=np.uint16).astype(np.uint8)
    raw[16:] = qs.tobytes()
    out = oracle.dequantize(synth.Q4_K, bytes(raw), 256)
    scales = [1, 2, 3, 4, 5, 6, 7, 8]
    for j in range(256):
        b = int(qs[j // 2])
        q = (b & 0xF) if j % 2 == 0 else (b >> 4)
        assert out[j] == np.float32(scales[j // 32] * q)
    # Q8_K: f32 d then 256 int8
    q8 = rng.integers(-128, 128, 256).astype(np.int8)
    raw = np.float32(0.25).tobytes() + q8.tobytes() + bytes(32)
    np.testing.assert_array_equal(oracle.dequantize(synth.Q8_K, raw, 256), np.float32(0.25) * q8.astype(np.float32))


# ---------------------------------------------------------------- IntegerMatMulTests.cs
def test_dot_int128(oracle):  # IntegerMatMulTests.cs:10-85
    assert oracle.dot_int128([3, 7], [5, 11]) == 92
    big = MAXL // 2
    assert oracle.dot_int128([big, big], [big, big]) == 2 * big * big
    assert oracle.dot_int128([-3, 7], [5, -11]) == -92
    assert oracle.dot_int128([0, 0, 0], [100, 200, 300]) == 0
    assert oracle.dot_int128([10**9], [10**9]) == 10**18
    assert oracle.dot_int128([99, 3, 7, 99][1:3], [99, 5, 11, 99][1:3]) == 92


def test_dot_int128_worst_case(oracle):  # IntegerMatMulTests.cs:337-387
    a = [1 << 30] * 768
    assert oracle.dot_int128(a, a) == 768 << 60
    alt = [(1 << 30) if i % 2 == 0 else -(1 << 30) for i in range(768)]
    assert oracle.dot_int128(alt, a) == 0


def test_matmul_known_results(oracle):  # IntegerMatMulTests.cs:87-159
    np.testing.assert_array_equal(oracle.matmul_long([1, 2, 3, 4], 2, 2, [1, 0, 0, 1], 2), [1, 2, 3, 4])
    np.testing.assert_array_equal(oracle.matmul_long([1, 2, 3], 1, 3, [4, 5, 6], 1), [32])
    a, w = [1, 2, 3, 4, 5, 6], [7, 8, 9, 10, 11, 12]
    np.testing.assert_array_equal(oracle.matmul_long(a, 2, 3, w, 2), [50, 68, 122, 167])
    np.testing.assert_array_equal(oracle.matmul_long(a, 2, 3, w, 2, shift=1), [25, 34, 61, 83])
    np.testing.assert_array_equal(oracle.matmul_long([-1, 2], 1, 2, [3, -4], 1), [-11])


def test_matmul_scaled_exponents(oracle):  # IntegerMatMulTests.cs:161-186
    assert oracle.matmul_long([100, 200], 1, 2, [3, 4], 1)[0] == 1100
    assert oracle.matmul_long([100, 200], 1, 2, [3, 4], 1, shift=5)[0] == 1100 >> 5


def test_right_shift_floors(oracle):  # IntegerMatMulTests.cs:188-198, 398-416
    # ScaledTensor.RightShift / RightShiftInPlace are `>>` on long: floor toward -inf.
    for v, s, e in [(1024, 3, 128), (-512, 3, -64), (7, 3, 0), (-1, 1, -1), (-3, 1, -2), (-7, 1, -4)]:
        assert oracle.matmul_long([v], 1, 1, [1], 1, shift=s)[0] == e


def test_quantize_from_float(oracle):  # IntegerMatMulTests.cs:200-232
    orig = np.array([0.5, -0.25, 0.125, 1.0, -1.0], np.float32)
    q = oracle.quantize_from_float(orig)
    assert np.abs(q / float(ONE) - orig).max() < 1e-6
    qa, qb = oracle.quantize_from_float(np.array([0.123456789, 0.123456780], np.float32))
    assert qa != qb


def test_matmul_matches_float(oracle):  # IntegerMatMulTests.cs:234-310
    a = np.array([0.1, 0.2, 0.3, 0.4, 0.5, 0.6], np.float32)
    w = np.array([0.7, 0.8, 0.9, 1.0, 1.1, 1.2], np.float32)
    c = oracle.matmul_long(oracle.quantize_from_float(a), 2, 3, oracle.quantize_from_float(w), 2)
    cf = (a.reshape(2, 3).astype(np.float64) @ w.reshape(2, 3).T.astype(np.float64)).reshape(-1)
    assert np.abs(c / float(1 << 60) - cf).max() < 1e-4
    rng = np.random.default_rng(42)
    dim, rows, cols = 768, 4, 768
    a = rng.uniform(-0.05, 0.05, rows * dim).astype(np.float32)
    w = rng.uniform(-0.05, 0.05, dim * cols).astype(np.float32)
    c = oracle.matmul_long(oracle.quantize_from_float(a), rows, dim, oracle.quantize_from_float(w), cols)
    cf = (a.reshape(rows, dim).astype(np.float64) @ w.reshape(cols, dim).T.astype(np.float64)).reshape(-1)
    m = np.abs(cf) > 1e-10
    assert (np.abs(c / float(1 << 60) - cf)[m] / np.abs(cf[m])).max() < 1e-3


def test_matmul_deterministic(oracle):  # IntegerMatMulTests.cs:312-335
    rng = np.random.default_rng(7)
    a = oracle.quantize_from_float(rng.uniform(-1, 1, 128).astype(np.float32))
    w = oracle.quantize_from_float(rng.uniform(-1, 1, 128 * 128).astype(np.float32))
    r0 = oracle.matmul_long(a, 1, 128, w, 128)
    for _ in range(10):
        np.testing.assert_array_equal(oracle.matmul_long(a, 1, 128, w, 128), r0)


# ---------------------------------------------------------------- IntegerLayerNormTests.cs
def test_isqrt64(oracle):  # IntegerLayerNormTests.cs:8-58
    for v, e in [(0, 0), (1, 1), (4, 2), (9, 3), (100, 10), (10**6, 1000), (10**12, 10**6),
                 (2, 1), (3, 1), (5, 2), (8, 2), (10, 3), (1 << 60, 1 << 30)]:
        assert oracle.isqrt64(v) == e
    r = oracle.isqrt64(MAXL)
    assert r * r <= MAXL < (r + 1) * (r + 1)
    for n in [0, 1, 2, 3, 4, 5, 7, 8, 9, 15, 16, 17, 99, 100, 101, 999_999, 10**6, 10**6 + 1,
              (1 << 50) - 1, 1 << 50, (1 << 50) + 1]:
        x = oracle.isqrt64(n)
        assert x >= 0 and x * x <= n and (x + 1) * (x + 1) > n


def test_isqrt128(oracle):  # IntegerLayerNormTests.cs:60-80
    for v, e in [(0, 0), (1, 1), (100, 10), (10**12, 10**6)]:
        assert oracle.isqrt128(v) == e
    big = 768 << 60
    r = oracle.isqrt128(big)
    assert r * r <= big < (r + 1) * (r + 1)
    rng = np.random.default_rng(5)
    for _ in range(200):
        v = int(rng.integers(1, 1 << 62)) * int(rng.integers(1, 1 << 62))
        r = oracle.isqrt128(v)
        assert r == math.isqrt(v)


def test_layernorm_known(oracle):  # IntegerLayerNormTests.cs:82-107, 228-268
    np.testing.assert_array_equal(oracle.layernorm([100] * 4, 1, 4, [ONE] * 4, [10, 20, 30, 40]), [10, 20, 30, 40])
    s = 1 << 20
    x = oracle.layernorm([-100 * s, 100 * s], 1, 2, [s, s], [0, 0])
    assert x[0] < 0 < x[1] and -x[0] == x[1]
    assert oracle.layernorm([500], 1, 1, [ONE], [42])[0] == 42
    x = oracle.layernorm([3 * s, 1 * s], 1, 2, [s, s], [0, 0])
    assert abs(x[0] - s) < s / 100 and abs(x[1] + s) < s / 100
    oracle.layernorm([1000000, 1000001, 1000000, 1000001], 1, 4, [ONE] * 4, [0] * 4)


def test_layernorm_matches_float(oracle):  # IntegerLayerNormTests.cs:109-200
    rng = np.random.default_rng(42)
    for seq in (1, 4):
        x = rng.uniform(-0.1, 0.1, seq * 768).astype(np.float32)
        w = rng.uniform(0.9, 1.1, 768).astype(np.float32)
        b = rng.uniform(-0.01, 0.01, 768).astype(np.float32)
        q = oracle.layernorm(oracle.quantize_from_float(x), seq, 768, oracle.quantize_from_float(w), oracle.quantize_from_float(b))
        xr = x.reshape(seq, 768).astype(np.float64)
        ref = (xr - xr.mean(1, keepdims=True)) / np.sqrt(xr.var(1, keepdims=True) + 1e-12) * w + b
        got = q.reshape(seq, 768) / float(ONE)
        m = np.abs(ref) > 1e-6
        assert (np.abs(got - ref)[m] / np.abs(ref[m])).max() < 0.05


def test_rmsnorm_uniform(oracle):  # IntegerLayerNormTests.cs:270-283
    s = 1 << 20
    x = oracle.rmsnorm([5 * s] * 4, 1, 4, [s] * 4)
    assert all(abs(v - s) < s / 100 for v in x)


# ---------------------------------------------------------------- IntegerAttentionTests.cs
def test_fixed_exp(oracle):  # IntegerAttentionTests.cs:10-54
    assert abs(oracle.fixed_exp(0) - ONE) / ONE < 1e-6
    assert abs(to_double(oracle.fixed_exp(ONE)) - math.e) / math.e < 1e-4
    for v in [-0.5, -1.0, -2.0, -5.0, -10.0]:
        got = to_double(oracle.fixed_exp(fixed_from_double(v)))
        assert abs(got - math.exp(v)) / math.exp(v) < 0.01
    assert oracle.fixed_exp(fixed_from_double(-50.0)) == 0


def test_fixed_sigmoid_silu(oracle):  # IntegerAttentionTests.cs:56-97
    assert abs(to_double(oracle.fixed_sigmoid(0)) - 0.5) < 0.01
    assert to_double(oracle.fixed_sigmoid(fixed_from_double(10.0))) > 0.999
    assert to_double(oracle.fixed_sigmoid(fixed_from_double(-10.0))) < 0.001
    for v in [-2.0, -1.0, -0.5, 0.0, 0.5, 1.0, 2.0]:
        got = to_double(oracle.fixed_silu(fixed_from_double(v)))
        assert abs(got - v / (1 + math.exp(-v))) < 0.02


def test_fixed_softmax(oracle):  # IntegerAttentionTests.cs:99-157, 277-309
    p = oracle.fixed_softmax([ONE] * 4)
    assert all(abs(to_double(v) - 0.25) < 0.01 for v in p)
    s = [fixed_from_double(v) for v in (2.0, 1.0, -1.0, 0.5)]
    p = oracle.fixed_softmax(s)
    assert abs(to_double(int(p.sum())) - 1.0) < 0.01
    f = np.array([2.0, 1.0, -1.0, 0.5])
    ref = np.exp(f - f.max()) / np.exp(f - f.max()).sum()
    assert (np.abs(p / float(ONE) - ref) / ref).max() < 0.02
    rng = np.random.default_rng(42)
    f = rng.uniform(-3, 3, 12)
    p = oracle.fixed_softmax([fixed_from_double(v) for v in f])
    ref = np.exp(f - f.max()) / np.exp(f - f.max()).sum()
    assert (np.abs(p / float(ONE) - ref) / ref).max() < 0.05


def test_rope_preserves_norm(oracle):  # IntegerAttentionTests.cs:159-191
    rng = np.random.default_rng(42)
    x = (np.trunc(rng.uniform(-100, 100, 64)).astype(np.int64) * (1 << 20))
    y = oracle.apply_rope(x, 1, 64, 2, 16, 32, 10000.0)
    nb = sum(int(v) * int(v) for v in x)
    na = sum(int(v) * int(v) for v in y)
    assert abs(na - nb) / nb < 0.01


def _rand_longs(rng, n, scale_bits):  # IntegerAttentionTests.cs:311-318
    m = 1 << (scale_bits - 2)
    return np.trunc(rng.uniform(-1, 1, n) * m).astype(np.int64)


def test_attention_small_deterministic(oracle):  # IntegerAttentionTests.cs:193-275
    rng = np.random.default_rng(42)
    q, k, v = (_rand_longs(rng, 24, 20) for _ in range(3))
    o1 = oracle.attention(q, k, v, 3, 8, 8, 2, 2, -20)
    assert o1.size == 24 and (o1 != 0).any()
    np.testing.assert_array_equal(o1, oracle.attention(q, k, v, 3, 8, 8, 2, 2, -20))
    q = _rand_longs(rng, 24, 20)
    k, v = _rand_longs(rng, 12, 20), _rand_longs(rng, 12, 20)
    g1 = oracle.attention(q, k, v, 3, 8, 4, 4, 2, -20)
    assert (g1 != 0).any()
    np.testing.assert_array_equal(g1, oracle.attention(q, k, v, 3, 8, 4, 4, 2, -20))


def test_sliding_window(oracle):  # IntegerAttentionTests.cs:320-397
    rng = np.random.default_rng(42)
    q, k, v = (_rand_longs(rng, 32, 20) for _ in range(3))
    full = oracle.attention(q, k, v, 4, 8, 8, 2, 2, -20, mode=1)
    sw = oracle.attention(q, k, v, 4, 8, 8, 2, 2, -20, mode=2, window=2)
    np.testing.assert_array_equal(full[:16], sw[:16])
    assert (full[24:] != sw[24:]).any()
    np.testing.assert_array_equal(full, oracle.attention(q, k, v, 4, 8, 8, 2, 2, -20, mode=2, window=104))


def test_causal_last_row_matches_noncausal(oracle):  # CausalModelProbeTests.cs:84-123
    rng = np.random.default_rng(42)
    q = rng.integers(-1000, 1000, 32)
    k, v = rng.integers(-1000, 1000, 16), rng.integers(-1000, 1000, 16)
    c = oracle.attention(q, k, v, 4, 8, 4, 2, 1, -20, mode=1)
    n = oracle.attention(q, k, v, 4, 8, 4, 2, 1, -20, mode=0)
    assert (c[:8] != 0).any()
    np.testing.assert_array_equal(c[24:], n[24:])
    np.testing.assert_array_equal(c, oracle.attention(q, k, v, 4, 8, 4, 2, 1, -20, mode=1))


def test_causal_mask_is_leaky(oracle):
    """maskValue = -(1 << (fracBits-1)) (IntegerAttention.cs:222): masked slots keep weight, so row 0
    of a causal head is not plain self-attention."""
    rng = np.random.default_rng(9)
    q, k, v = (rng.integers(-(1 << 30), 1 << 30, 8) for _ in range(3))
    c = oracle.attention(q, k, v, 2, 4, 4, 1, 1, -30, mode=1)
    assert (c[:4] != v[:4]).any()


# ---- lattice k-NN search ----

def test_quantize_kills_noise_under_threshold(oracle):  # EmbeddingAdapterTests.cs:8-22
    q = oracle.quantize_dense(np.array([0.0, 0.005, -0.005, 0.5, -0.8, 0.001], np.float32), 0.01, (1 << 63) - 1)
    assert (q != 0).sum() == 2 and q[3] != 0 and q[4] != 0


def test_quantize_defaults_sign_and_zeros(oracle):  # EmbeddingAdapterTests.cs:24-50
    big = (1 << 63) - 1
    assert (oracle.quantize_dense(np.array([0.0, 0.005, -0.005], np.float32), 0.01, big) == 0).all()
    q = oracle.quantize_dense(np.array([0.0, 0.5, -0.5], np.float32), 0.01, big)
    assert q[0] == 0 and q[1] > 0 and q[2] < 0


def test_quantize_truncates_double_product(oracle):
    """(long)(e * (double)GlobalScale): the float widens to double, the product rounds once, the cast
    truncates toward zero; NaN and out-of-range give long.MinValue."""
    e = np.array([0.1, -0.1, 0.3333333, 1e-3, 0.0009999, 2.5, np.nan], np.float32)
    q = oracle.quantize_dense(e, 0.001, 1_000_000_000)
    expect = [int(np.float64(np.float32(x)) * 1e9) if np.isfinite(x) and abs(x) >= np.float32(0.001) else 0 for x in e[:-1]]
    assert list(q[:-1]) == expect
    assert q[-1] == np.iinfo(np.int64).min
    assert oracle.quantize_dense(np.array([1.0], np.float32), 0.0, (1 << 63) - 1)[0] == np.iinfo(np.int64).min


def test_distance_squared_l2_known(oracle):  # SparseVectorTests.cs:103-116, 118-136
    a = np.array([10, 0, 30, 0, 0], np.int64)
    b = np.array([7, 20, 25, 0, 0], np.int64)
    assert oracle.distance_sq_l2_fast(a, b) == 434
    a = np.array([10, 0, 30, 0, 5], np.int64)
    assert oracle.distance_sq_l2_fast(a, b) == sum((int(x) - int(y)) ** 2 for x, y in zip(a, b))
    assert oracle.distance_sq_l2_fast(a, a) == 0  # SparseVectorTests.cs:207-214


def test_distance_fast_wraps_in_ulong(oracle):
    """DistanceSquaredL2Fast sums (ulong)(diff * diff) with long wrap-around (SparseVector.cs:138-169)."""
    a = np.array([3_000_000_000, 3_000_000_000], np.int64)
    b = np.array([0, -3_000_000_000], np.int64)
    exact = 3_000_000_000 ** 2 + 6_000_000_000 ** 2
    assert oracle.distance_sq_l2_fast(a, b) == exact % (1 << 64)


def test_knn_linear_items(oracle):  # KnnQueryTests.cs:14-22, 92-102 (BuildLinearItems :277-286)
    db = np.zeros((5, 5), np.int64)
    db[:, 0] = (np.arange(5) + 1) * 100
    center = np.array([[300, 0, 0, 0, 0]], np.int64)
    ids, dist = oracle.knn_l2(db, center, 100)
    assert (ids[0, :5] >= 0).all() and (ids[0, 5:] == -1).all()  # k > corpus: all 5 rows, then padding
    assert list(ids[0, :5]) == [2, 1, 3, 0, 4]  # equal distances (1 and 3) ordered by id
    assert list(dist[0, :5]) == [0, 10000, 10000, 40000, 40000]
    ids0, _ = oracle.knn_l2(db, center, 0)
    assert ids0.shape == (1, 0)


def test_knn_matches_sorted_brute_force(oracle):  # KnnQueryTests.cs:75-90 (RecallEvaluator.BruteForceKNearestL2)
    rng = np.random.default_rng(7)
    db = np.zeros((60, 8), np.int64)
    db[:, :2] = rng.integers(100, 1000, (60, 2))
    center = np.zeros((1, 8), np.int64)
    center[0, 0], center[0, 2] = 400, 600
    ids, dist = oracle.knn_l2(db, center, 5)
    full = sorted((oracle.distance_sq_l2_fast(center[0], db[r]), r) for r in range(60))
    assert [r for _, r in full[:5]] == list(ids[0]) and [d for d, _ in full[:5]] == list(dist[0])
