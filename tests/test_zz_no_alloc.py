"""The allocation-free projection GEMM, slx_matmul_q30_noalloc, against slx_matmul_q30_device.

slx_matmul_q30_noalloc serves callers that must not allocate device memory: services whose GPU
memory is owned by another allocator (so a cudaMalloc inside a request fails or breaks the budget)
and latency-bound request paths that cannot pay for cudaMalloc. Its scratch is a fixed array inside
the library. Here the test owns the inputs and outputs (allocated with torch), calls both entry
points through the C ABI on the same stream, and requires identical int64 results -- the products
are exact integers, so the tolerance is zero -- on two calls in a row, the second with other
shapes and an activation too wide for the tensor-core digits, so the shared scratch is reused.
This file is collected last so a failure here cannot hide the other tests' results.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_noalloc_matches_device_entry_point_on_two_calls():
    import torch

    import spatialdb_b200 as slx
    from spatialdb_b200 import _lib, synth

    lib = _lib.lib()
    ctx = slx.Context(0)
    torch.cuda.set_device(0)
    stream = torch.cuda.Stream()
    h = ctypes.c_void_p(stream.cuda_stream)
    rng = np.random.default_rng(2024)
    cases = [(200, 512, 192, synth.Q8_0, False), (130, 768, 256, synth.Q4_0, True)]
    for call, (M, K, N, dtype, wide) in enumerate(cases):
        raw = synth.random_q8_0(rng, N * K) if dtype == synth.Q8_0 else synth.random_q4_0(rng, N * K)
        a = rng.integers(-(1 << 36), 1 << 36, (M, K), dtype=np.int64)
        if wide:
            a[M - 1, K - 1] = 1 << 50  # beyond 5 digits: the call must take the exact kernel
        d_a = torch.from_numpy(a).cuda()
        d_w = torch.from_numpy(raw).cuda()
        ref = torch.empty((M, N), dtype=torch.int64, device="cuda")
        got = torch.full((M, N), -7, dtype=torch.int64, device="cuda")
        torch.cuda.synchronize()
        st = lib.slx_matmul_q30_device(ctx._h, ctypes.c_void_p(d_a.data_ptr()), M, K, dtype,
                                       ctypes.c_void_p(d_w.data_ptr()), raw.size, N, 0, 30, 30,
                                       ctypes.c_void_p(ref.data_ptr()), h)
        assert st == 0, lib.slx_last_error(ctx._h)
        st = lib.slx_matmul_q30_noalloc(ctypes.c_void_p(d_a.data_ptr()), M, K, dtype, ctypes.c_void_p(d_w.data_ptr()),
                                        raw.size, N, 0, 30, 30, ctypes.c_void_p(got.data_ptr()), h)
        assert st == 0, f"call {call}: status {st}"
        stream.synchronize()
        assert torch.equal(ref, got), f"call {call}: outputs differ"


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
