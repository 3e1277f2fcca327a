// k_gemm_tc.cu -- exact Q30 projection GEMM on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// IntegerMatMul.MatMul (Math/IntegerMatMul.cs:37-76) needs sum_k a[m][k]*w[n][k] exactly (Int128)
// before the >> 30. Both operands are split into balanced base-256 digits in [-128, 127]:
//     a = sum_i a_i 256^i  (LA = 5 digits: |a| < ~2^39),   w = sum_j w_j 256^j  (LW <= 4 digits),
// so  sum_k a w = sum_s 256^s P_s  with  P_s = sum_{i+j=s} sum_k a_ik w_jk.
// Each P_s is an exact int32 (|a_i w_j| <= 2^14, at most 4 pairs per s, K < 32768) and
// accumulates in TMEM. One tcgen05.mma.kind::i8 per activation digit i and 32-wide K step uses the
// weight digit planes stacked along N (LW x 64 rows) as the B operand and writes its accumulator at
// TMEM column offset 64*i: the product a_i*w_j lands in column block i+j, so all pairs of equal
// shift s sum in the same TMEM columns (S = LA+LW-1 blocks of 64 columns, <= 512).
// The epilogue combines the S int32 partials per output into Int128, applies the shift (floor) and
// the optional residual, and stores int64 -- bit-identical to the reference.
//
// Operands arrive by TMA (cp.async.bulk.tensor, 128-byte swizzle, no multicast) into a 2-stage
// smem ring; one thread issues the MMAs; tcgen05.commit releases ring stages and signals the
// epilogue. Every mbarrier wait is bounded: on timeout the kernel records an error, waits
// (bounded) for its outstanding copies, frees TMEM and returns.
#include <cuda.h>

#include <cstring>

#include "slx_device.cuh"
#include "slx_gemm.h"
#include "slx_kernels.h"
#include "tc_ptx.cuh"

namespace slx {
namespace tc {

// BM = 128 output rows per CTA (TMEM lanes), BN = 64 output columns, BK = 128 K bytes per ring
// stage (one 128-byte swizzle row), LA = 5 activation digits (slx_gemm.h).
constexpr int THREADS = 192;

struct Params {
    int M, N, K, nkb, lw, shift, nstages;
    int64_t* C;
    int64_t ldc;
    const int64_t* R;
    int64_t ldr;
    const int* skip;  // nonzero: an operand did not fit its digits, the exact kernel runs instead
    int* err;         // set on a bounded-wait timeout
    // the weight row n was stored as w >> row_shift[n] (its common trailing zeros)
    const int8_t* row_shift;
};

template <int LW, int BN>
__global__ void __launch_bounds__(THREADS, 1)
k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW, Params p) {
    constexpr int S = LA + LW - 1;
    static_assert(S * BN <= 512, "TMEM holds 512 columns");
    static_assert((BN * LW) % 16 == 0 && BN * LW <= 256, "M=128 MMA needs N a multiple of 16, at most 256");
    constexpr int A_STAGE = BM * BK * LA;
    constexpr int W_STAGE = BN * BK * LW;
    constexpr int STAGE = A_STAGE + W_STAGE;
    constexpr uint32_t IDESC = idesc_i8(BN * LW);
    if (p.skip && *p.skip) return;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int nst = p.nstages;
    uint64_t* bars = (uint64_t*)(smem + (size_t)nst * STAGE);
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + nst), done = smem_u32(bars + 2 * nst);
    uint32_t* tmem_slot = (uint32_t*)(bars + 2 * nst + 1);
    __shared__ int s_fail;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        s_fail = 0;
        for (int i = 0; i < nst; i++) {
            mbar_init(full0 + 8 * i, 1);
            mbar_init(empty0 + 8 * i, 1);
        }
        mbar_init(done, 1);
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

    // Zero the accumulators: digit products of different i overlap in their column blocks, so every
    // MMA accumulates.
    if (warp >= 2) {
        const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
#pragma unroll
        for (int c = 0; c < S * BN; c += 16) tmem_st16_zero(tmem + lane_base + c);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    fence_before();
    __syncthreads();
    fence_after();

    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const uint32_t sbase = smem_u32(smem);

    if (warp == 0) {
        if (lane == 0) {  // TMA producer
            int issued = 0;
            for (int kb = 0; kb < p.nkb; kb++) {
                const int s = kb % nst;
                const uint32_t ph = (uint32_t)(kb / nst) & 1u;
                if (!mbar_wait(empty0 + 8 * s, ph ^ 1u)) { s_fail = 1; break; }
                if (*(volatile int*)&s_fail) break;
                mbar_expect_tx(full0 + 8 * s, STAGE);
                tma_load_4d(sbase + s * STAGE, &tmA, kb * BK, m0, 0, 0, full0 + 8 * s);
                tma_load_4d(sbase + s * STAGE + A_STAGE, &tmW, kb * BK, n0, 0, 0, full0 + 8 * s);
                issued = kb + 1;
            }
            if (*(volatile int*)&s_fail) {  // let copies still in flight land before the CTA exits
                for (int kb = issued - nst < 0 ? 0 : issued - nst; kb < issued; kb++)
                    mbar_wait(full0 + 8 * (kb % nst), (uint32_t)(kb / nst) & 1u);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            for (int kb = 0; kb < p.nkb; kb++) {
                const int s = kb % nst;
                const uint32_t ph = (uint32_t)(kb / nst) & 1u;
                if (!mbar_wait(full0 + 8 * s, ph)) { s_fail = 1; break; }
                fence_after();
                const uint32_t a = sbase + s * STAGE, w = a + A_STAGE;
#pragma unroll
                for (int kk = 0; kk < BK / 32; kk++) {
                    const uint64_t bdesc = sw128_desc(w + kk * 32);
#pragma unroll
                    for (int i = 0; i < LA; i++)
                        umma_i8(tmem + i * BN, sw128_desc(a + i * (BM * BK) + kk * 32), bdesc, IDESC, 1u);
                }
                umma_commit(empty0 + 8 * s);
            }
            umma_commit(done);
        }
    } else {  // epilogue: warps 2..5, TMEM lanes 32*(warp%4) ..
        const bool ok = __all_sync(0xffffffffu, mbar_wait(done, 0));  // tcgen05.ld below is warp-collective
        if (!ok) s_fail = 1;
        fence_after();
        const int lb = 32 * (warp & 3);
        const int row = m0 + lb + lane;
        const uint32_t taddr = tmem + ((uint32_t)lb << 16);
        if (ok) {
#pragma unroll 1
            for (int c = 0; c < BN / 16; c++) {
                uint32_t v[S][16];
#pragma unroll
                for (int s = 0; s < S; s++) tmem_ld16(taddr + s * BN + c * 16, v[s]);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (row < p.M) {
                    int64_t* crow = p.C + (int64_t)row * p.ldc;
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const int n = n0 + c * 16 + j;
                        if (n >= p.N) break;
                        i128 acc = (i128)(int32_t)v[S - 1][j];
#pragma unroll
                        for (int s = S - 2; s >= 0; s--) acc = (acc << 8) + (i128)(int32_t)v[s][j];
                        if (p.row_shift) acc <<= p.row_shift[n];
                        int64_t out = p.shift > 0 ? lo64(sar128(acc, p.shift)) : lo64(acc);
                        if (p.R) out = wadd(out, p.R[(int64_t)row * p.ldr + n]);
                        crow[n] = out;
                    }
                }
            }
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

// Balanced base-256 digits of activations: planes[i][m][k] (m < Mpad, k < Kpad, zero padded).
// Sets *overflow when a value needs more than LA digits.
__global__ void k_split_a(const int64_t* __restrict__ A, int64_t lda, int M, int K, int Mpad, int Kpad,
                          int8_t* __restrict__ planes, int* overflow) {
    const int chunks = Kpad / 16;
    const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (idx >= (int64_t)Mpad * chunks) return;
    const int row = (int)(idx / chunks), k0 = (int)(idx % chunks) * 16;
    uint32_t pk[LA][4];
#pragma unroll
    for (int i = 0; i < LA; i++)
#pragma unroll
        for (int q = 0; q < 4; q++) pk[i][q] = 0;
    bool bad = false;
#pragma unroll
    for (int j = 0; j < 16; j++) {
        int64_t x = (row < M && k0 + j < K) ? A[(int64_t)row * lda + k0 + j] : 0;
#pragma unroll
        for (int i = 0; i < LA; i++) {
            int d = (int)(((uint64_t)x + 128u) & 255u) - 128;
            x = (x - d) >> 8;
            pk[i][j >> 2] |= (uint32_t)(uint8_t)(int8_t)d << (8 * (j & 3));
        }
        bad |= x != 0;
    }
    if (bad) atomicOr(overflow, 1);
#pragma unroll
    for (int i = 0; i < LA; i++)
        *(uint4*)(planes + ((int64_t)i * Mpad + row) * Kpad + k0) = make_uint4(pk[i][0], pk[i][1], pk[i][2], pk[i][3]);
}

// Balanced digits of per-head rows: X row (b*T + t), head h, hd values at X + (b*T+t)*ld + h*hd
// -> planes[(b*nh + h)][i][t][k] (t < tpad, k < kpad, zero padded). Sets *overflow when a value
// needs more than LA digits.
__global__ void k_split_heads(const int64_t* __restrict__ X, int64_t ld, int T, int nh, int hd, int tpad, int kpad,
                              int8_t* __restrict__ planes, int* overflow, int64_t total) {
    const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (idx >= total) return;
    const int chunks = kpad / 16;
    const int k0 = (int)(idx % chunks) * 16;
    const int64_t r = idx / chunks;  // over (b*nh + h) * tpad + t
    const int t = (int)(r % tpad);
    const int64_t bh = r / tpad;
    const int h = (int)(bh % nh);
    const int64_t b = bh / nh;
    uint32_t pk[LA][4];
#pragma unroll
    for (int i = 0; i < LA; i++)
#pragma unroll
        for (int q = 0; q < 4; q++) pk[i][q] = 0;
    bool bad = false;
#pragma unroll
    for (int j = 0; j < 16; j++) {
        int64_t x = (t < T && k0 + j < hd) ? X[(b * T + t) * ld + (int64_t)h * hd + k0 + j] : 0;
#pragma unroll
        for (int i = 0; i < LA; i++) {
            int d = (int)(((uint64_t)x + 128u) & 255u) - 128;
            x = (x - d) >> 8;
            pk[i][j >> 2] |= (uint32_t)(uint8_t)(int8_t)d << (8 * (j & 3));
        }
        bad |= x != 0;
    }
    if (bad) atomicOr(overflow, 1);
#pragma unroll
    for (int i = 0; i < LA; i++)
        *(uint4*)(planes + ((bh * LA + i) * tpad + t) * kpad + k0) = make_uint4(pk[i][0], pk[i][1], pk[i][2], pk[i][3]);
}

// Common trailing zero bits of each weight row's Q30 composites (0 for an all-zero row).
// Q4_0 / Q8_0 composites are d_int * q with d_int an f16 mantissa times a power of two, so a row
// typically shares ten or more low zero bits; storing w >> tz[n] saves one or two digits.
__global__ void k_weight_tz(WDesc W, int8_t* tz) {
    const int n = blockIdx.x;
    int m = 64;
    for (int64_t k = threadIdx.x; k < W.K; k += blockDim.x) {
        int64_t x = composite(dequant_elem(W.dtype, W.data, (int64_t)n * W.K + k, W.nblocks), W.mode, W.scale);
        if (x != 0) m = min(m, __ffsll(x) - 1);
    }
    for (int o = 16; o > 0; o >>= 1) m = min(m, __shfl_xor_sync(0xffffffffu, m, o));
    __shared__ int sm[32];
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 1; i < (int)(blockDim.x >> 5); i++) m = min(m, sm[i]);
        m = min(m, sm[0]);
        tz[n] = (int8_t)(m >= 63 ? 0 : m);
    }
}

// Number of balanced base-256 digits the largest (row-shifted) composite weight needs.
__global__ void k_weight_digits(WDesc W, int* maxd, const int8_t* tz) {
    int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    int nd = 0;
    if (e < W.N * W.K) {
        int64_t x = composite(dequant_elem(W.dtype, W.data, e, W.nblocks), W.mode, W.scale);
        if (tz) x >>= tz[e / W.K];
        while (x != 0 && nd < 9) {
            int d = (int)(((uint64_t)x + 128u) & 255u) - 128;
            x = (x - d) >> 8;
            nd++;
        }
    }
    for (int o = 16; o > 0; o >>= 1) nd = max(nd, __shfl_xor_sync(0xffffffffu, nd, o));
    if ((threadIdx.x & 31) == 0 && nd) atomicMax(maxd, nd);
}

// Weight digit planes[j][n][k] (n < Npad, k < Kpad, zero padded) of the Q30 composite, shifted
// right by the row's common trailing zeros when tz is given.
__global__ void k_split_w(WDesc W, int lw, int Npad, int Kpad, int8_t* __restrict__ planes, const int8_t* tz) {
    const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (idx >= (int64_t)Npad * Kpad) return;
    const int n = (int)(idx / Kpad), k = (int)(idx % Kpad);
    int64_t x = (n < W.N && k < W.K) ? composite(dequant_elem(W.dtype, W.data, (int64_t)n * W.K + k, W.nblocks), W.mode, W.scale) : 0;
    if (tz && n < W.N) x >>= tz[n];
    for (int j = 0; j < lw; j++) {
        int d = (int)(((uint64_t)x + 128u) & 255u) - 128;
        x = (x - d) >> 8;
        planes[((int64_t)j * Npad + n) * Kpad + k] = (int8_t)d;
    }
}

// ---------------------------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------------------------
namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                  const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    }
    return fn;
}

template <int LW, int BNT>
constexpr size_t stage_bytes() { return (size_t)BM * BK * LA + (size_t)BNT * BK * LW; }

template <int LW, int BNT>
int stages() {
    int n = (int)((227 * 1024 - 1024 - 256) / stage_bytes<LW, BNT>());
    return n > 4 ? 4 : n;
}

template <int LW, int BNT>
void launch_lw(const CUtensorMap& ta, const CUtensorMap& tw, Params p, dim3 grid, cudaStream_t st) {
    p.nstages = stages<LW, BNT>();
    const size_t smem = p.nstages * stage_bytes<LW, BNT>() + 1024 + (2 * p.nstages + 2) * 8;
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(k_gemm_tc<LW, BNT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        configured = true;
    }
    k_gemm_tc<LW, BNT><<<grid, THREADS, smem, st>>>(ta, tw, p);
}

Params base_params() {
    Params p;
    memset(&p, 0, sizeof p);
    return p;
}
}  // namespace

bool encode_planes(void* map128, void* base, int64_t kpad, int64_t rows, int planes, int box_rows, int64_t batch) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || kpad % BK || planes < 1 || planes > 255 || box_rows < 1 || box_rows > 256 || batch < 1) return false;
    if (((uintptr_t)base & 15) != 0) return false;
    cuuint64_t dims[4] = {(cuuint64_t)kpad, (cuuint64_t)rows, (cuuint64_t)planes, (cuuint64_t)batch};
    cuuint64_t strides[3] = {(cuuint64_t)kpad, (cuuint64_t)(kpad * rows), (cuuint64_t)(kpad * rows * planes)};
    cuuint32_t box[4] = {(cuuint32_t)BK, (cuuint32_t)box_rows, (cuuint32_t)planes, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn((CUtensorMap*)map128, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, base, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool encode_rows_u16(void* map128, const void* base, int64_t row_u16, int64_t rows, int box_x, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || box_x < 8 || box_x > 256 || (box_x * 2) % 16 || box_rows < 1 || box_rows > 256) return false;
    if (((uintptr_t)base & 15) != 0 || (row_u16 * 2) % 16 != 0) return false;
    cuuint64_t dims[2] = {(cuuint64_t)row_u16, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(row_u16 * 2)};
    cuuint32_t box[2] = {(cuuint32_t)box_x, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn((CUtensorMap*)map128, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box,
                    estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

void weight_tz(const WDesc& w, int8_t* tz, cudaStream_t st) {
    k_weight_tz<<<(unsigned)w.N, 256, 0, st>>>(w, tz);
}

int weight_digits(const WDesc& w, cudaStream_t st, std::string& err, const int8_t* tz) {
    int* d_max = nullptr;
    if (cudaMalloc(&d_max, sizeof(int)) != cudaSuccess) { err = "device allocation failed"; return -1; }
    cudaMemsetAsync(d_max, 0, sizeof(int), st);
    const int64_t n = w.N * w.K;
    k_weight_digits<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(w, d_max, tz);
    int maxd = 0;
    cudaMemcpyAsync(&maxd, d_max, sizeof(int), cudaMemcpyDeviceToHost, st);
    cudaError_t e = cudaStreamSynchronize(st);
    cudaFree(d_max);
    if (e != cudaSuccess) { err = cudaGetErrorString(e); return -1; }
    return maxd;
}

void split_w(const WDesc& w, int lw, int64_t npad, int64_t kpad, int8_t* planes, cudaStream_t st, const int8_t* tz) {
    const int64_t tot = npad * kpad;
    k_split_w<<<(unsigned)((tot + 255) / 256), 256, 0, st>>>(w, lw, (int)npad, (int)kpad, planes, tz);
}

void split_a(const int64_t* a, int64_t lda, int M, int K, int64_t mpad, int64_t kpad, int8_t* planes, int* overflow,
             cudaStream_t st) {
    const int64_t chunks = mpad * (kpad / 16);
    k_split_a<<<(unsigned)((chunks + 255) / 256), 256, 0, st>>>(a, lda, M, K, (int)mpad, (int)kpad, planes, overflow);
}

void launch(const void* tmap_a, const void* tmap_w, int lw, int M, int N, int K, int64_t mpad, int64_t npad, int64_t kpad,
            int shift, int64_t* c, int64_t ldc, const int64_t* r, int64_t ldr, const int* skip, int* err, cudaStream_t st,
            const int8_t* row_shift) {
    Params p = base_params();
    p.M = M; p.N = N; p.K = K; p.nkb = (int)(kpad / BK); p.lw = lw; p.shift = shift; p.nstages = 2;
    p.C = c; p.ldc = ldc; p.R = r; p.ldr = ldr; p.skip = skip; p.err = err; p.row_shift = row_shift;
    dim3 grid((unsigned)(npad / BN), (unsigned)(mpad / BM));
    const CUtensorMap& ta = *(const CUtensorMap*)tmap_a;
    const CUtensorMap& tw = *(const CUtensorMap*)tmap_w;
    switch (lw) {
        case 1: launch_lw<1, BN>(ta, tw, p, grid, st); break;
        case 2: launch_lw<2, BN>(ta, tw, p, grid, st); break;
        case 3: launch_lw<3, BN>(ta, tw, p, grid, st); break;
        default: launch_lw<4, BN>(ta, tw, p, grid, st); break;
    }
}

void split_heads(const int64_t* x, int64_t ld, int B, int T, int nh, int hd, int64_t tpad, int64_t kpad, int8_t* planes,
                 int* overflow, cudaStream_t st) {
    const int64_t total = (int64_t)B * nh * tpad * (kpad / 16);
    if (total <= 0) return;
    k_split_heads<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(x, ld, T, nh, hd, (int)tpad, (int)kpad, planes, overflow,
                                                                  total);
}


}  // namespace tc
}  // namespace slx
