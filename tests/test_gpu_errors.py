"""Device-side error reporting, without a GPU fault.

* A tensor-core projection GEMM whose pipeline waits run out: the context option
  SLX_OPT_TEST_STALL_MMA keeps the kernel's MMA warp idle, so the TMA producer's wait for a free
  stage and the epilogue's wait for a finished accumulator can never complete; with a short
  SLX_OPT_WAIT_LIMIT_CYCLES they give up after about a millisecond, the kernel lets its copies land,
  frees its tensor memory and returns, and the call reports SLX_ETIMEOUT. The same context then
  computes the next call correctly.
* slx_encode_device queues work without waiting, so the errors its kernels raise (a bounded-wait
  timeout, a token id whose UNK row lies outside the table) are read afterwards with
  slx_ctx_status, which reports them once and clears them.
Nothing here faults, traps or hangs a GPU: every wait is bounded and ends with a status the host
reads.
"""
import os

import numpy as np
import pytest

import spatialdb_b200 as slx
from spatialdb_b200 import synth

pytestmark = pytest.mark.gpu

SHORT_WAIT = 2_000_000  # SM clock cycles: about a millisecond at 1.9 GHz


def _oracle_matmul(oracle, a, raw, N):
    M, K = a.shape
    f = oracle.dequantize(synth.Q8_0, raw, N * K)
    return oracle.matmul_long(a, M, K, oracle.quantize_from_float(f), N, 30).reshape(M, N)


def test_gemm_wait_timeout_reports_and_context_recovers(oracle):
    ctx = slx.Context(0)
    rng = np.random.default_rng(11)
    M, K, N = 64, 512, 256  # M > 8: the tensor-core GEMM, not the decode GEMV
    raw = synth.random_q8_0(rng, N * K)
    a = rng.integers(-(1 << 36), 1 << 36, (M, K), dtype=np.int64)
    ctx.set_option(slx.OPT_WAIT_LIMIT_CYCLES, SHORT_WAIT)
    ctx.set_option(slx.OPT_TEST_STALL_MMA, 1)
    with pytest.raises(slx.SlxError) as e:
        slx.matmul_q30(a, synth.Q8_0, raw, N, ctx=ctx)
    assert e.value.status == slx.SLX_ETIMEOUT, str(e.value)
    ctx.set_option(slx.OPT_TEST_STALL_MMA, 0)
    ctx.set_option(slx.OPT_WAIT_LIMIT_CYCLES, 0)
    got = slx.matmul_q30(a, synth.Q8_0, raw, N, ctx=ctx)
    np.testing.assert_array_equal(got, _oracle_matmul(oracle, a, raw, N))


@pytest.fixture(scope="module")
def small_encoder(tmpdir_session):
    shape = synth.EncoderShape(layers=2, embd=64, heads=4, ff=128, vocab=500, ctx=512)
    ok = synth.write_encoder(os.path.join(tmpdir_session, "err_enc.gguf"), shape, synth.Q8_0, seed=8)
    bad_unk = synth.write_encoder(os.path.join(tmpdir_session, "err_enc_unk.gguf"), shape, synth.Q8_0, seed=8,
                                  unk=shape.vocab + 10)
    return shape, ok, bad_unk


def _encode_device(model, ids, stream):
    import torch

    d_ids = torch.from_numpy(ids).cuda()
    pooled = torch.empty((ids.shape[0], model.embd), dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()
    model.encode_device(d_ids.data_ptr(), ids.shape[0], ids.shape[1], pooled.data_ptr(), stream.cuda_stream)
    return d_ids, pooled


def test_encode_device_reports_timeout_through_ctx_status(oracle, small_encoder):
    import torch

    shape, path, _ = small_encoder
    ctx = slx.Context(0)
    stream = torch.cuda.Stream()
    m = slx.IntegerTransformerSource.load(path, ctx=ctx)
    ids = np.random.default_rng(3).integers(0, shape.vocab, (2, 40)).astype(np.int32)
    ctx.set_option(slx.OPT_WAIT_LIMIT_CYCLES, SHORT_WAIT)
    ctx.set_option(slx.OPT_TEST_STALL_MMA, 1)
    _encode_device(m, ids, stream)
    with pytest.raises(slx.SlxError) as e:
        ctx.status(stream.cuda_stream)
    assert e.value.status == slx.SLX_ETIMEOUT, str(e.value)
    ctx.set_option(slx.OPT_TEST_STALL_MMA, 0)
    ctx.set_option(slx.OPT_WAIT_LIMIT_CYCLES, 0)
    ctx.status(stream.cuda_stream)  # cleared by the first read
    _, pooled = _encode_device(m, ids, stream)
    ctx.status(stream.cuda_stream)
    np.testing.assert_array_equal(pooled.cpu().numpy(), oracle.Encoder(path).forward(ids))


def test_encode_device_reports_out_of_range_ids_through_ctx_status(oracle, small_encoder):
    import torch

    shape, path, bad_unk = small_encoder
    ctx = slx.Context(0)
    stream = torch.cuda.Stream()
    m = slx.IntegerTransformerSource.load(bad_unk, ctx=ctx)
    ids = np.random.default_rng(4).integers(0, shape.vocab, (2, 16)).astype(np.int32)
    bad = ids.copy()
    bad[1, 5] = shape.vocab + 3  # past the table, and the UNK row is past it too
    _encode_device(m, bad, stream)
    with pytest.raises(slx.IndexOutOfRangeError):
        ctx.status(stream.cuda_stream)
    with pytest.raises(slx.IndexOutOfRangeError):  # the host-buffer entry point checks by itself
        m.forward(bad)
    _, pooled = _encode_device(m, ids, stream)  # in-range ids never read the UNK row
    ctx.status(stream.cuda_stream)
    np.testing.assert_array_equal(pooled.cpu().numpy(), oracle.Encoder(bad_unk).forward(ids))
