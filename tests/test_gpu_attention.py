"""Attention parity (IntegerAttention) of the tensor-core score path and the exact fallback."""
import os
import subprocess
import sys

import numpy as np
import pytest

import spatialdb_b200 as slx

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def ctx():
    return slx.Context(0)


def _qkv(rng, seq, qe, kve, mag):
    return (rng.integers(-mag, mag, (seq, qe), dtype=np.int64), rng.integers(-mag, mag, (seq, kve), dtype=np.int64),
            rng.integers(-mag, mag, (seq, kve), dtype=np.int64))


@pytest.mark.parametrize("seq,nh,nkv,hd", [(1, 4, 4, 64), (7, 4, 4, 64), (64, 12, 12, 64), (130, 2, 2, 64),
                                           (512, 2, 2, 64), (33, 8, 1, 256), (200, 4, 2, 32), (70, 3, 3, 16)])
@pytest.mark.parametrize("mode,window", [(0, 0), (1, 0), (2, 5)])
def test_attention_matches_oracle(ctx, oracle, seq, nh, nkv, hd, mode, window):
    rng = np.random.default_rng(seq * 31 + nh * 7 + hd + mode)
    q, k, v = _qkv(rng, seq, nh * hd, nkv * hd, 1 << 32)
    got = slx.attention(q, k, v, seq, nh, nkv, -30, mode, window, ctx=ctx)
    ref = oracle.attention(q, k, v, seq, nh * hd, nkv * hd, nh, nkv, -30, 30, mode, window).reshape(seq, nh * hd)
    np.testing.assert_array_equal(got, ref)


def test_attention_reference_test_shapes(ctx, oracle):
    """The reference tests' shapes (IntegerAttentionTests.cs:193-275, 320-397): scaleBits 20, hd 4."""
    rng = np.random.default_rng(42)
    m = 1 << 18
    for seq, qe, kve, nh, nkv, mode, win in [(3, 8, 8, 2, 2, 0, 0), (3, 8, 4, 4, 2, 0, 0), (4, 8, 8, 2, 2, 1, 0),
                                             (4, 8, 8, 2, 2, 2, 2), (4, 8, 4, 2, 1, 1, 0)]:
        q, k, v = _qkv(rng, seq, qe, kve, m)
        got = slx.attention(q, k, v, seq, nh, nkv, -20, mode, win, ctx=ctx)
        ref = oracle.attention(q, k, v, seq, qe, kve, nh, nkv, -20, 30, mode, win).reshape(seq, qe)
        np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("hd", [16, 64, 256])
def test_attention_values_at_the_fp64_window_edge(ctx, oracle, hd):
    """|v| up to the P.V's bound 2^50 (the accumulator window [2^52, 2^53) holds every partial sum),
    with rows at both ends of the range; one value at 2^50 sends the call to the exact kernel."""
    rng = np.random.default_rng(11 + hd)
    seq, nh = 150, 3
    q, k, _ = _qkv(rng, seq, nh * hd, nh * hd, 1 << 32)
    v = rng.integers(-(1 << 50), 1 << 50, (seq, nh * hd), dtype=np.int64)
    v[0, :] = (1 << 50) - 1
    v[1, :] = -(1 << 50)
    v[2, ::2] = (1 << 50) - 1
    for mode in (0, 1):
        got = slx.attention(q, k, v, seq, nh, nh, -30, mode, 0, ctx=ctx)
        ref = oracle.attention(q, k, v, seq, nh * hd, nh * hd, nh, nh, -30, 30, mode, 0).reshape(seq, nh * hd)
        np.testing.assert_array_equal(got, ref)
    v[7, 5] = 1 << 50
    got = slx.attention(q, k, v, seq, nh, nh, -30, 0, 0, ctx=ctx)
    ref = oracle.attention(q, k, v, seq, nh * hd, nh * hd, nh, nh, -30, 30, 0, 0).reshape(seq, nh * hd)
    np.testing.assert_array_equal(got, ref)


def test_attention_one_hot_softmax(ctx, oracle):
    """One key dominates every row: p = 2^30 for it and 0 elsewhere, so each product p v / 2^30 is an
    exact integer (the directed rounding must not move it)."""
    rng = np.random.default_rng(5)
    seq, nh, hd = 70, 2, 64
    q = np.full((seq, nh * hd), 1 << 33, np.int64)
    k = rng.integers(-(1 << 10), 1 << 10, (seq, nh * hd), dtype=np.int64)
    k[3, :] = 1 << 33
    v = rng.integers(-(1 << 45), 1 << 45, (seq, nh * hd), dtype=np.int64)
    got = slx.attention(q, k, v, seq, nh, nh, -30, 0, 0, ctx=ctx)
    ref = oracle.attention(q, k, v, seq, nh * hd, nh * hd, nh, nh, -30, 30, 0, 0).reshape(seq, nh * hd)
    np.testing.assert_array_equal(got, ref)
    np.testing.assert_array_equal(ref, np.broadcast_to(v[3], ref.shape))


@pytest.mark.parametrize("what", ["q_wide", "k_wide", "v_wide", "scores_wrap"])
def test_attention_out_of_range_inputs_fall_back_exactly(ctx, oracle, what):
    rng = np.random.default_rng(9)
    seq, nh, hd = 96, 2, 64
    q, k, v = _qkv(rng, seq, nh * hd, nh * hd, 1 << 31)
    if what == "q_wide":
        q[5, 3] = 1 << 45
    elif what == "k_wide":
        k[17, 100] = -(1 << 50)
    elif what == "v_wide":
        v[3, 7] = np.iinfo(np.int64).max
    else:  # scores spanning more than 2^63 wrap in the reference's long subtraction
        q[0, :] = 1 << 38
        k[:, :] = rng.integers(-(1 << 38), 1 << 38, k.shape)
    got = slx.attention(q, k, v, seq, nh, nh, -30, 1, 0, ctx=ctx)
    ref = oracle.attention(q, k, v, seq, nh * hd, nh * hd, nh, nh, -30, 30, 1, 0).reshape(seq, nh * hd)
    np.testing.assert_array_equal(got, ref)


def test_exact_kernels_alone_match_oracle():
    """With the tensor-core paths disabled (SLX_DISABLE_TC=1) the exact CUDA-core kernels carry the
    whole forward; run the encoder and causal parity tests that way in a child process."""
    env = dict(os.environ, SLX_DISABLE_TC="1")
    r = subprocess.run([sys.executable, "-m", "pytest", "-x", "-q", "-m", "gpu", os.path.join(ROOT, "tests", "test_gpu_parity.py"),
                        "-k", "encoder_layers or causal_forward or gemma_encoder"], env=env, capture_output=True, text=True,
                       timeout=900, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
