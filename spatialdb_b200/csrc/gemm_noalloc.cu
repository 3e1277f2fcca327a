// gemm_noalloc.cu -- the projection GEMM for callers that must not allocate device memory.
//
// Who needs it: a host service whose GPU memory is owned by another allocator (a framework's
// caching allocator or a pre-sized arena that has reserved the free HBM), where a cudaMalloc from
// inside a request either fails or breaks the memory budget, and latency-bound request paths
// that cannot afford cudaMalloc's cost and implicit device synchronisation. slx_matmul_q30_device
// allocates the weight's digit planes and its activation workspace per call; this variant puts all
// of that scratch in one fixed device array compiled into the library instead.
//
// The scratch is a file-scope __device__ array of SLX_NOALLOC_SCRATCH_BYTES (32 MiB). Every GPU
// that loads libslx holds it until the process exits. In host code the array's name is only a
// host-side stand-in, not a device address: its address on each device is looked up once per
// device with cudaGetSymbolAddress (the first call of the entry point on a device does that, with
// the device current) and passed to the kernels.
//
// All calls share the array and it keeps the last call's contents: the overflow and error words
// are cleared at the start of each call, and every plane byte the kernels read is rewritten by
// the call. Calls whose GPU work overlaps (different streams, or different host threads on one
// device) race on the array and must be serialised by the caller.
#include <cuda_runtime.h>

#include <mutex>

#include "slx.h"
#include "slx_device.cuh"
#include "slx_gemm.h"
#include "slx_kernels.h"

namespace slx {
namespace {

constexpr size_t kScratchBytes = (size_t)SLX_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;
constexpr int kWeightDigits = 4;  // fixed: weights needing more digits raise the overflow word

// Scratch layout: [0, 4) overflow word, [64, 68) error word, planes from byte 256.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_addr[kMaxDevices];  // device address of g_noalloc_scratch, per device ordinal

// Device address of the scratch array on the current device (looked up once per device).
cudaError_t scratch_on_current_device(uint8_t** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_addr[dev] = p;
    }
    *out = (uint8_t*)g_scratch_addr[dev];
    return cudaSuccess;
}

// Weight digit planes [4][npad][kpad] of the Q30 composites; raises *overflow when a composite
// needs more than 4 balanced digits (the exact kernel then computes the call).
__global__ void k_split_w_checked(WDesc W, int npad, int kpad, int8_t* __restrict__ planes, int* overflow) {
    const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (idx >= (int64_t)npad * kpad) return;
    const int n = (int)(idx / kpad), k = (int)(idx % kpad);
    int64_t x = (n < W.N && k < W.K)
                    ? composite(dequant_elem(W.dtype, W.data, (int64_t)n * W.K + k, W.nblocks), W.mode, W.scale)
                    : 0;
#pragma unroll
    for (int j = 0; j < kWeightDigits; j++) {
        int d = (int)(((uint64_t)x + 128u) & 255u) - 128;
        x = (x - d) >> 8;
        planes[((int64_t)j * npad + n) * kpad + k] = (int8_t)d;
    }
    if (x != 0) atomicOr(overflow, 1);
}

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

}  // namespace
}  // namespace slx

using namespace slx;

extern "C" slx_status slx_matmul_q30_noalloc(const int64_t* d_a, int M, int K, int dtype, const uint8_t* d_w,
                                             int64_t w_bytes, int N, int half_composite, int scale_bits, int shift,
                                             int64_t* d_c, void* stream) {
    if (M <= 0 || K <= 0 || N <= 0 || !d_a || !d_w || !d_c || scale_bits < 1 || scale_bits > 62) return SLX_EINVAL;
    if (dtype != DT_F32 && dtype != DT_F16 && dtype != DT_BF16 && dtype != DT_Q8_0 && dtype != DT_Q4_0)
        return SLX_EUNSUPPORTED;
    const int64_t elems = (int64_t)N * K;
    const int64_t need_w = dtype == DT_Q8_0 ? (elems / 32) * 34
                         : dtype == DT_Q4_0 ? (elems / 32) * 18
                         : (dtype == DT_F32 ? elems * 4 : elems * 2);
    if (w_bytes < need_w) return SLX_EEOF;
    const int64_t mpad = round_up(M, tc::BM), npad = round_up(N, tc::BN), kpad = round_up(K, tc::BK);
    const int64_t a_bytes = round_up((int64_t)tc::LA * mpad * kpad, 256);
    const int64_t w_planes = (int64_t)kWeightDigits * npad * kpad;
    if (K >= 32768 || 256 + a_bytes + w_planes > (int64_t)kScratchBytes) return SLX_ESCRATCH;

    uint8_t* scratch = nullptr;
    if (scratch_on_current_device(&scratch) != cudaSuccess) return SLX_ECUDA;
    cudaStream_t st = (cudaStream_t)stream;
    int* overflow = (int*)scratch;
    int* err = (int*)(scratch + 64);
    int8_t* a_planes = (int8_t*)(scratch + 256);
    int8_t* w_dig = a_planes + a_bytes;

    WDesc w;
    w.dtype = dtype; w.data = d_w; w.nblocks = elems / 32; w.elements = elems; w.N = N; w.K = K;
    w.mode = half_composite ? 1 : 0;
    w.scale = ldexp(1.0, scale_bits);

    alignas(64) unsigned char map_a[128], map_w[128];
    if (!tc::encode_planes(map_a, a_planes, kpad, mpad, tc::LA, tc::GM, 1, tc::GK) ||
        !tc::encode_planes(map_w, w_dig, kpad, npad, kWeightDigits, tc::GN, 1, tc::GK))
        return SLX_ECUDA;
    if (cudaMemsetAsync(scratch, 0, 256, st) != cudaSuccess) return SLX_ECUDA;  // overflow and error words
    const int64_t tot = npad * kpad;
    k_split_w_checked<<<(unsigned)((tot + 255) / 256), 256, 0, st>>>(w, (int)npad, (int)kpad, w_dig, overflow);
    tc::split_a(d_a, K, M, K, mpad, kpad, a_planes, overflow, st);
    // (the exact product runs in the same launch if a value overflowed its digits)
    tc::launch(map_a, map_w, kWeightDigits, M, N, K, mpad, npad, kpad, shift, d_c, N, nullptr, 0, overflow, err, st, nullptr,
               nullptr, d_a, K, &w);
    if (cudaGetLastError() != cudaSuccess) return SLX_ECUDA;
    int host_err = 0;
    if (cudaMemcpyAsync(&host_err, err, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess) return SLX_ECUDA;
    if (cudaStreamSynchronize(st) != cudaSuccess) return SLX_ECUDA;
    return host_err ? SLX_ETIMEOUT : SLX_OK;
}
