// k_fgemm_tc.cu -- the float twin's projections on the tensor cores: C = A . W^T in fp32 with the
// operands split as x = x_hi + x_lo (x_hi: x with its low 13 mantissa bits cleared, exactly a tf32
// value; x_lo = x - x_hi, exact in fp32) and three tf32 products per pair, A_hi W_hi + A_hi W_lo +
// A_lo W_hi, accumulated in fp32 by tcgen05.mma.kind::tf32 (the dropped A_lo W_lo is below 2^-21
// of the product). The reference's float encoder (Gguf/TransformerEmbeddingSource.cs) sums its
// products in fp32 Vector<float> lanes in a machine-dependent order, so this path, like the FFMA
// kernel it replaces for the projections, is held to a tolerance against the oracle.
//
// Layout: weights are split once at load into planes [2][N][Kp] (hi, lo; Kp = K rounded up to 32
// floats, the padding zero), activations per call into [2][M][Kp]. A CTA tile is 128 weight rows
// (the MMA's M, TMEM lanes) x 256 activation rows (its N); K moves in stages of 32 floats (one
// 128-byte swizzled row per operand row and plane, by 4D TMA without multicast): 96 KB a stage,
// two stages. Per 8-float K step three MMAs into the tile's fp32 accumulator (256 TMEM columns; two
// accumulators, so the epilogue of one tile overlaps the next tile's MMAs). The epilogue thread of
// weight row n writes C[m][n] for its 64 activation rows: a warp stores 32 consecutive n of a row.
// Persistent: one CTA per SM walks the tiles, weight tiles fastest. Every mbarrier wait is bounded.
#include <cuda.h>

#include <algorithm>

#include "slx_attr.h"
#include "slx_float.h"
#include "slx_gemm.h"
#include "tc_ptx.cuh"

namespace slx {
namespace fenc {
namespace {

using namespace tc;

constexpr int FM = 128;            // weight rows per tile (MMA M)
constexpr int FN = 256;            // activation rows per tile (MMA N)
constexpr int FKB = 128;           // bytes of K per stage and row (32 floats)
constexpr int FST = 2;             // stages
constexpr int FEPI = 16;           // epilogue warps: four per TMEM lane quarter, 64 activation rows each
constexpr int FTHREADS = 32 * (2 + FEPI);
constexpr int W_ST = 2 * FM * FKB, A_ST = 2 * FN * FKB, F_STAGE = W_ST + A_ST;
constexpr size_t F_SMEM = (size_t)FST * F_STAGE + 1024 + 256;
static_assert(F_SMEM <= 227 * 1024, "fp32 projection tiles");

// Instruction descriptor, kind::tf32: D f32, A and B tf32, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_tf32(int n) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}
__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

struct FParams {
    int M, N, nkb, tiles_n, tiles;
    float* C;
    int64_t ldc;
    int* err;
};

// Split x into (hi, lo) planes of [rows][Kp] (zero from K to Kp); non-finite values keep x in hi.
__global__ void k_split_tf32(const float* __restrict__ x, int64_t ldx, int rows, int K, int Kp, float* __restrict__ hi,
                             float* __restrict__ lo) {
    const int64_t total = (int64_t)rows * Kp;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / Kp), k = (int)(i % Kp);
        const float v = k < K ? x[(int64_t)r * ldx + k] : 0.0f;
        float h = v, l = 0.0f;
        if (isfinite(v)) {
            h = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
            l = v - h;
        }
        hi[i] = h;
        lo[i] = l;
    }
}

__global__ void __launch_bounds__(FTHREADS, 1)
k_fgemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW, FParams p) {
    constexpr uint32_t IDESC = idesc_tf32(FN);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = (uint64_t*)(smem + (size_t)FST * F_STAGE);
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + FST);
    const uint32_t tfull0 = smem_u32(bars + 2 * FST), tfree0 = smem_u32(bars + 2 * FST + 2);
    const uint32_t drain = smem_u32(bars + 2 * FST + 4);
    uint32_t* tmem_slot = (uint32_t*)(bars + 2 * FST + 5);
    __shared__ int s_fail;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        s_fail = 0;
        for (int i = 0; i < FST; i++) {
            mbar_init(full0 + 8 * i, 1);
            mbar_init(empty0 + 8 * i, 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(tfull0 + 8 * b, 1);
            mbar_init(tfree0 + 8 * b, FEPI);
        }
        mbar_init(drain, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t sbase = smem_u32(smem);

    if (warp == 0) {
        if (lane == 0) {  // TMA producer, running ahead across tiles
            int g = 0, s = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < p.tiles; t += gridDim.x) {
                const int m0 = (t / p.tiles_n) * FN, n0 = (t % p.tiles_n) * FM;
                for (int kb = 0; kb < p.nkb; kb++, g++) {
                    if (!mbar_wait(empty0 + 8 * s, ph ^ 1u) || *(volatile int*)&s_fail) {
                        s_fail = 1;
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(full0 + 8 * s, F_STAGE);
                    tma_load_4d(sbase + s * F_STAGE, &tmW, kb * FKB, n0, 0, 0, full0 + 8 * s);
                    tma_load_4d(sbase + s * F_STAGE + W_ST, &tmA, kb * FKB, m0, 0, 0, full0 + 8 * s);
                    if (++s == FST) { s = 0; ph ^= 1u; }
                }
            }
            if (!ok)  // let copies still in flight land before the CTA exits (they always complete)
                for (int j = g - FST < 0 ? 0 : g - FST; j < g; j++) mbar_wait(full0 + 8 * (j % FST), (uint32_t)(j / FST) & 1u);
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            int lt = 0, s = 0;
            uint32_t ph = 0;
            bool ok = true, issued = false;
            for (int t = blockIdx.x; ok && t < p.tiles; t += gridDim.x, lt++) {
                const int b = lt & 1;
                if (!mbar_wait(tfree0 + 8 * b, ((uint32_t)(lt >> 1) & 1u) ^ 1u)) { ok = false; break; }
                fence_after();
                const uint32_t d = tmem + b * FN;
                for (int kb = 0; kb < p.nkb; kb++) {
                    if (!mbar_wait(full0 + 8 * s, ph)) { ok = false; break; }
                    fence_after();
                    const uint32_t w = sbase + s * F_STAGE, a = w + W_ST;
#pragma unroll
                    for (int kk = 0; kk < FKB / 32; kk++) {
                        const uint64_t whi = sw128_desc(w + kk * 32), wlo = sw128_desc(w + FM * FKB + kk * 32);
                        const uint64_t ahi = sw128_desc(a + kk * 32), alo = sw128_desc(a + FN * FKB + kk * 32);
                        umma_tf32(d, whi, ahi, IDESC, kb == 0 && kk == 0 ? 0u : 1u);
                        umma_tf32(d, whi, alo, IDESC, 1u);
                        umma_tf32(d, wlo, ahi, IDESC, 1u);
                    }
                    umma_commit(empty0 + 8 * s);
                    issued = true;
                    if (++s == FST) { s = 0; ph ^= 1u; }
                }
                if (!ok) break;
                umma_commit(tfull0 + 8 * b);
            }
            if (!ok) {
                s_fail = 1;
                if (issued) {  // MMAs still in flight write TMEM: let them retire before it is freed
                    umma_commit(drain);
                    mbar_wait(drain, 0u);
                }
            }
        }
    } else {  // epilogue: thread = weight row (TMEM lane), 64 of the tile's activation rows
        const int q4 = warp & 3, part = (warp - 2) >> 2;
        const uint32_t lane_base = (uint32_t)(32 * q4) << 16;
        int lt = 0;
        for (int t = blockIdx.x; t < p.tiles; t += gridDim.x, lt++) {
            const int b = lt & 1;
            const int m0 = (t / p.tiles_n) * FN, n0 = (t % p.tiles_n) * FM;
            const int n = n0 + 32 * q4 + lane;
            if (!__all_sync(0xffffffffu, mbar_wait(tfull0 + 8 * b, (uint32_t)(lt >> 1) & 1u))) {
                s_fail = 1;
                break;
            }
            fence_after();
#pragma unroll 1
            for (int c = 0; c < 64; c += 16) {
                uint32_t v[16];
                tmem_ld16(tmem + lane_base + b * FN + 64 * part + c, v);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (n < p.N) {
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const int m = m0 + 64 * part + c + j;
                        if (m < p.M) p.C[(int64_t)m * p.ldc + n] = __uint_as_float(v[j]);
                    }
                }
            }
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tfree0 + 8 * b);
        }
    }
    fence_before();
    __syncthreads();
    if (s_fail && threadIdx.x == 0 && p.err) atomicOr(p.err, KERR_TIMEOUT);
    if (warp == 1) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
    }
}

int64_t kpad_of(int K) { return (K + 31) / 32 * 32; }
}  // namespace

size_t tc_weight_bytes(int N, int K) { return (size_t)2 * N * kpad_of(K) * sizeof(float); }

bool tc_prepare_weight(const float* w, int N, int K, float* planes, cudaStream_t st) {
    if (N <= 0 || K <= 0) return false;
    const int64_t kp = kpad_of(K);
    const int64_t total = (int64_t)N * kp;
    const unsigned grid = (unsigned)std::min<int64_t>((total + 255) / 256, 148 * 16);
    k_split_tf32<<<grid, 256, 0, st>>>(w, K, N, K, (int)kp, planes, planes + total);
    return cudaGetLastError() == cudaSuccess;
}

size_t tc_act_bytes(int M, int K) { return (size_t)2 * M * kpad_of(K) * sizeof(float); }

bool tc_project(const float* a, int M, int K, const float* w_planes, int N, float* c, float* act_planes, int* err,
                cudaStream_t st) {
    if (M <= 0 || N <= 0 || K <= 0) return false;
    const int64_t kp = kpad_of(K);
    alignas(64) unsigned char mapA[128], mapW[128];
    if (!tc::encode_planes(mapA, act_planes, kp * 4, M, 2, FN, 1, FKB) ||
        !tc::encode_planes(mapW, const_cast<float*>(w_planes), kp * 4, N, 2, FM, 1, FKB))
        return false;
    const int64_t total = (int64_t)M * kp;
    const unsigned sgrid = (unsigned)std::min<int64_t>((total + 255) / 256, 148 * 16);
    k_split_tf32<<<sgrid, 256, 0, st>>>(a, K, M, K, (int)kp, act_planes, act_planes + total);
    if (slx::ensure_smem((const void*)k_fgemm_tc, F_SMEM) != cudaSuccess) return false;
    FParams p;
    p.M = M; p.N = N; p.nkb = (int)(kp * 4 / FKB);
    p.tiles_n = (N + FM - 1) / FM;
    p.tiles = p.tiles_n * ((M + FN - 1) / FN);
    p.C = c; p.ldc = N; p.err = err;
    CUtensorMap ta, tw;
    memcpy(&ta, mapA, sizeof(ta));
    memcpy(&tw, mapW, sizeof(tw));
    const int grid = std::min(p.tiles, slx::device_sm_count());
    k_fgemm_tc<<<grid, FTHREADS, F_SMEM, st>>>(ta, tw, p);
    return cudaGetLastError() == cudaSuccess;
}

}  // namespace fenc
}  // namespace slx
