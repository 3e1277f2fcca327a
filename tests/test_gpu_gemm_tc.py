"""Parity of the tensor-core projection GEMM (balanced int8 digits on tcgen05) with the oracle.

Activations are drawn inside the 5-digit range (|a| < 2^38) so the tensor-core path produces the
result; the overflow cases push one activation outside it, which must route that call to the
exact CUDA-core kernel with the same bit-exact answer.
"""
import numpy as np
import pytest

import spatialdb_b200 as slx
from spatialdb_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    return slx.Context(0)


def _raw(dtype, rng, n):
    if dtype == synth.Q8_0:
        return synth.random_q8_0(rng, n)
    if dtype == synth.Q4_0:
        return synth.random_q4_0(rng, n)
    return synth.encode(dtype, rng.standard_normal(n).astype(np.float32) * 0.05)


def _ref(oracle, a, dtype, raw, N, half, shift):
    M, K = a.shape
    f = oracle.dequantize(dtype, raw, N * K)
    if half:
        return oracle.matmul_half(a, M, K, oracle.float_to_half(f), N, 30, shift).reshape(M, N)
    return oracle.matmul_long(a, M, K, oracle.quantize_from_float(f), N, shift).reshape(M, N)


@pytest.mark.parametrize("M,K,N", [(1, 128, 64), (128, 128, 64), (200, 384, 130), (256, 768, 2304), (300, 3072, 768),
                                   (129, 96, 70)])
@pytest.mark.parametrize("dtype,half", [(synth.Q8_0, False), (synth.Q4_0, False), (synth.Q4_0, True), (synth.F16, False)])
def test_tc_matches_oracle(ctx, oracle, M, K, N, dtype, half):
    rng = np.random.default_rng(M + 7 * K + 13 * N + dtype)
    raw = _raw(dtype, rng, N * K)
    a = rng.integers(-(1 << 37), 1 << 37, (M, K), dtype=np.int64)
    for shift in (30, 0):
        got = slx.matmul_q30(a, dtype, raw, N, half_composite=half, shift=shift, ctx=ctx)
        np.testing.assert_array_equal(got, _ref(oracle, a, dtype, raw, N, half, shift), err_msg=f"shift {shift}")


def test_tc_digit_edges(ctx, oracle):
    """Activations at the digit boundaries (+-128, +-2^31, the 5-digit limits) and all-zero rows."""
    rng = np.random.default_rng(3)
    M, K, N = 160, 256, 96
    raw = _raw(synth.Q8_0, rng, N * K)
    edges = np.array([127, 128, -128, -129, 255, 256, -256, 1 << 31, -(1 << 31), (1 << 38) + 12345,
                      -(1 << 38) - 999, 0, 1, -1], np.int64)
    a = rng.choice(edges, size=(M, K))
    a[5] = 0
    got = slx.matmul_q30(a, synth.Q8_0, raw, N, ctx=ctx)
    np.testing.assert_array_equal(got, _ref(oracle, a, synth.Q8_0, raw, N, False, 30))


@pytest.mark.parametrize("big", [1 << 45, np.iinfo(np.int64).min, np.iinfo(np.int64).max])
def test_tc_overflow_falls_back_exactly(ctx, oracle, big):
    rng = np.random.default_rng(4)
    M, K, N = 130, 256, 64
    raw = _raw(synth.Q4_0, rng, N * K)
    a = rng.integers(-(1 << 30), 1 << 30, (M, K), dtype=np.int64)
    a[77, 13] = big
    got = slx.matmul_q30(a, synth.Q4_0, raw, N, ctx=ctx)
    np.testing.assert_array_equal(got, _ref(oracle, a, synth.Q4_0, raw, N, False, 30))


def test_tc_exact_integer_weights(ctx):
    """F32 weights v * 2^-30 have composite exactly v, so c = a . w^T in plain integers (shift 0)."""
    M, K, N = 128, 128, 64
    a = np.eye(M, K, dtype=np.int64)
    w = np.array([[n * 1000 + k for k in range(K)] for n in range(N)], np.int64)
    raw = (w.astype(np.float64) * 2.0 ** -30).astype(np.float32).reshape(-1).view(np.uint8)
    got = slx.matmul_q30(a, synth.F32, raw, N, shift=0, ctx=ctx)
    np.testing.assert_array_equal(got, a @ w.T)


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8])
@pytest.mark.parametrize("dtype", [synth.Q4_0, synth.Q8_0])
@pytest.mark.parametrize("K,N", [(64, 37), (4096, 300), (1024, 1030)])
def test_gemv_matches_oracle(ctx, oracle, M, dtype, K, N):
    """Decode-shaped calls (M <= 8, long composite) take the packed-block GEMV."""
    rng = np.random.default_rng(M * 131 + K + N + dtype)
    raw = _raw(dtype, rng, N * K)
    a = rng.integers(-(1 << 37), 1 << 37, (M, K), dtype=np.int64)
    got = slx.matmul_q30(a, dtype, raw, N, shift=30, ctx=ctx)
    np.testing.assert_array_equal(got, _ref(oracle, a, dtype, raw, N, False, 30))


@pytest.mark.parametrize("M", [1, 2])
def test_gemv_non_finite_scales_and_overflow(ctx, oracle, M):
    rng = np.random.default_rng(77)
    K, N = 256, 40
    raw = synth.random_q4_0(rng, N * K).reshape(-1, 18)
    raw[3, 0:2] = np.frombuffer(np.float16(np.inf).tobytes(), np.uint8)
    raw[9, 0:2] = np.frombuffer(np.float16(np.nan).tobytes(), np.uint8)
    raw[11, 0:2] = np.frombuffer(np.float16(-np.inf).tobytes(), np.uint8)
    raw = raw.reshape(-1)
    a = rng.integers(-(1 << 30), 1 << 30, (M, K), dtype=np.int64)
    np.testing.assert_array_equal(slx.matmul_q30(a, synth.Q4_0, raw, N, ctx=ctx), _ref(oracle, a, synth.Q4_0, raw, N, False, 30))
    a[M - 1, 5] = 1 << 44  # beyond 5 digits: exact fallback
    np.testing.assert_array_equal(slx.matmul_q30(a, synth.Q4_0, raw, N, ctx=ctx), _ref(oracle, a, synth.Q4_0, raw, N, False, 30))


@pytest.mark.parametrize("K,N", [(8192, 70), (2048, 1001), (256, 5)])
@pytest.mark.parametrize("dtype", [synth.Q4_0, synth.Q8_0])
def test_gemv_single_row_widths(ctx, oracle, K, N, dtype):
    """M = 1 at the single-row kernel's limits: 256 quant blocks a row (one row group per CTA), row
    counts that leave a partial last stage, rows narrower than a warp of blocks, and activations at
    the five-digit limits."""
    rng = np.random.default_rng(K + N + dtype)
    raw = _raw(dtype, rng, N * K)
    a = rng.integers(-(1 << 38), 1 << 38, (1, K), dtype=np.int64)
    a[0, :3] = [0x7F7F7F7F7F, -0x8080808080, 0]
    for shift in (30, 0):
        got = slx.matmul_q30(a, dtype, raw, N, shift=shift, ctx=ctx)
        np.testing.assert_array_equal(got, _ref(oracle, a, dtype, raw, N, False, shift))


@pytest.mark.parametrize("M", [1, 3, 8])
@pytest.mark.parametrize("dtype", [synth.Q4_0, synth.Q8_0])
def test_gemv_split_k_uneven(ctx, oracle, M, dtype):
    """K = 11008 (43 chunks of 256, split unevenly over the CTAs along K) and N with a ragged last
    row tile: the Int128 partials of every row tile add up exactly."""
    K, N = 11008, 200
    rng = np.random.default_rng(M * 17 + dtype)
    raw = _raw(dtype, rng, N * K)
    a = rng.integers(-(1 << 38), 1 << 38, (M, K), dtype=np.int64)
    for shift in (30, 0):
        got = slx.matmul_q30(a, dtype, raw, N, shift=shift, ctx=ctx)
        np.testing.assert_array_equal(got, _ref(oracle, a, dtype, raw, N, False, shift))


def test_gemv_large_scale_bits_take_general_path(ctx, oracle):
    """scale_bits beyond 39 can push d * q * 2^s past 2^63 (long.MinValue composites): the general
    path handles them; the result still matches the reference's composites."""
    rng = np.random.default_rng(12)
    K, N = 512, 64
    raw = synth.random_q8_0(rng, N * K)
    a = rng.integers(-(1 << 20), 1 << 20, (2, K), dtype=np.int64)
    f = oracle.dequantize(synth.Q8_0, raw, N * K)
    w = np.array([int(x) for x in (f.astype(np.float64) * 2.0 ** 45)], dtype=object)
    w = np.array([v if -(1 << 63) <= v < (1 << 63) else -(1 << 63) for v in w], np.int64)
    want = oracle.matmul_long(a, 2, K, w, N, 30).reshape(2, N)
    got = slx.matmul_q30(a, synth.Q8_0, raw, N, scale_bits=45, shift=30, ctx=ctx)
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("M", [1, 8, 128, 200])
@pytest.mark.parametrize("dtype,half", [(synth.Q8_0, False), (synth.Q4_0, False), (synth.Q4_0, True)])
def test_prepared_weight_matches_oracle(ctx, oracle, M, dtype, half):
    """slx_weight_prepare + slx_matmul_q30_prepared: digit planes built once, several products."""
    import torch

    rng = np.random.default_rng(31 * M + dtype)
    K, N = 512, 384
    raw = _raw(dtype, rng, N * K)
    d_w = torch.from_numpy(raw).cuda()
    w = slx.PreparedWeight(d_w.data_ptr(), raw.size, dtype, N, K, half_composite=half, ctx=ctx)
    assert (w.N, w.K) == (N, K) and w.tensor_cores == 1
    stream = torch.cuda.Stream()
    for rep in range(2):
        a = rng.integers(-(1 << 37), 1 << 37, (M, K), dtype=np.int64)
        d_a = torch.from_numpy(a).cuda()
        d_c = torch.empty((M, N), dtype=torch.int64, device="cuda")
        torch.cuda.synchronize()
        w.matmul_device(d_a.data_ptr(), M, d_c.data_ptr(), stream=stream.cuda_stream)
        ctx.status(stream.cuda_stream)
        np.testing.assert_array_equal(d_c.cpu().numpy(), _ref(oracle, a, dtype, raw, N, half, 30), err_msg=f"rep {rep}")
    w.close()
