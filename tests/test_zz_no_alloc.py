"""The allocation-free projection GEMM, slx_matmul_q30_noalloc, against the oracle.

slx_matmul_q30_noalloc serves callers that must not allocate device memory: services whose GPU
memory is owned by another allocator (so a cudaMalloc inside a request fails or breaks the budget)
and latency-bound request paths that cannot pay for cudaMalloc. Its scratch is a fixed array inside
the library. Here the test owns the inputs and outputs (allocated with torch), calls the entry
point through the C ABI several times in a row on one stream, so the shared scratch is reused with
other shapes, and requires the int64 results to equal the oracle's IntegerMatMul bit for bit (the
products are exact integers, so the tolerance is zero) and to equal slx_matmul_q30_device's. The
calls cover an activation too wide for the tensor-core digits, weights whose composites need more
than the scratch path's four weight digits (both routed to the exact kernel), and a decode-shaped
call (M <= 8), for which slx_matmul_q30_device takes its GEMV kernels instead.
This file is collected last so a failure here cannot hide the other tests' results.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _oracle_matmul(oracle, a, dtype, raw, N, half, shift):
    M, K = a.shape
    f = oracle.dequantize(dtype, raw, N * K)
    if half:
        return oracle.matmul_half(a, M, K, oracle.float_to_half(f), N, 30, shift).reshape(M, N)
    return oracle.matmul_long(a, M, K, oracle.quantize_from_float(f), N, shift).reshape(M, N)


def test_noalloc_matches_oracle_on_calls_in_a_row(oracle):
    import torch

    import spatialdb_b200 as slx
    from spatialdb_b200 import _lib, synth

    lib = _lib.lib()
    ctx = slx.Context(0)
    torch.cuda.set_device(0)
    stream = torch.cuda.Stream()
    h = ctypes.c_void_p(stream.cuda_stream)
    rng = np.random.default_rng(2024)
    # (M, K, N, dtype, half composite, what the call exercises)
    cases = [(200, 512, 192, synth.Q8_0, False, "tensor cores"),
             (130, 768, 256, synth.Q4_0, True, "wide activation"),
             (96, 256, 80, synth.F32, False, "wide weights"),
             (4, 512, 128, synth.Q4_0, False, "decode shape")]
    for call, (M, K, N, dtype, half, what) in enumerate(cases):
        if dtype == synth.Q8_0:
            raw = synth.random_q8_0(rng, N * K)
        elif dtype == synth.Q4_0:
            raw = synth.random_q4_0(rng, N * K)
        else:  # |f| up to 8: composites (long)(f * 2^30) need five balanced base-256 digits
            f = (rng.standard_normal(N * K) * 0.05).astype(np.float32)
            f[::7] = rng.uniform(-8, 8, f[::7].size).astype(np.float32)
            raw = synth.encode(dtype, f)
        a = rng.integers(-(1 << 36), 1 << 36, (M, K), dtype=np.int64)
        if what == "wide activation":
            a[M - 1, K - 1] = 1 << 50  # beyond 5 digits: the call must take the exact kernel
        want = _oracle_matmul(oracle, a, dtype, raw, N, half, 30)
        d_a = torch.from_numpy(a).cuda()
        d_w = torch.from_numpy(raw).cuda()
        ref = torch.empty((M, N), dtype=torch.int64, device="cuda")
        got = torch.full((M, N), -7, dtype=torch.int64, device="cuda")
        torch.cuda.synchronize()
        st = lib.slx_matmul_q30_noalloc(ctypes.c_void_p(d_a.data_ptr()), M, K, dtype, ctypes.c_void_p(d_w.data_ptr()),
                                        raw.size, N, int(half), 30, 30, ctypes.c_void_p(got.data_ptr()), h)
        assert st == 0, f"call {call} ({what}): status {st}"
        st = lib.slx_matmul_q30_device(ctx._h, ctypes.c_void_p(d_a.data_ptr()), M, K, dtype,
                                       ctypes.c_void_p(d_w.data_ptr()), raw.size, N, int(half), 30, 30,
                                       ctypes.c_void_p(ref.data_ptr()), h)
        assert st == 0, lib.slx_last_error(ctx._h)
        stream.synchronize()
        np.testing.assert_array_equal(got.cpu().numpy(), want, err_msg=f"call {call} ({what}) vs the oracle")
        assert torch.equal(ref, got), f"call {call} ({what}): differs from slx_matmul_q30_device"


def test_noalloc_rejects_requests_beyond_its_scratch():
    import torch

    import spatialdb_b200 as slx
    from spatialdb_b200 import _lib, synth

    lib = _lib.lib()
    M, K, N = 4096, 4096, 64  # 5 * 4096 * 4096 bytes of activation digits > 32 MiB
    d_a = torch.zeros((M, K), dtype=torch.int64, device="cuda")
    d_w = torch.zeros(synth.block_bytes(synth.Q8_0, N * K), dtype=torch.uint8, device="cuda")
    c = torch.zeros((M, N), dtype=torch.int64, device="cuda")
    st = lib.slx_matmul_q30_noalloc(ctypes.c_void_p(d_a.data_ptr()), M, K, synth.Q8_0, ctypes.c_void_p(d_w.data_ptr()),
                                    d_w.numel(), N, 0, 30, 30, ctypes.c_void_p(c.data_ptr()), None)
    assert st == slx.SLX_ESCRATCH
