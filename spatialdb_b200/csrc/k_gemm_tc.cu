// k_gemm_tc.cu -- exact Q30 projection GEMM on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// IntegerMatMul.MatMul (Math/IntegerMatMul.cs:37-76) needs sum_k a[m][k]*w[n][k] exactly (Int128)
// before the >> 30. Both operands are split into balanced base-256 digits in [-128, 127]:
//     a = sum_i a_i 256^i  (LA = 5 digits: |a| < ~2^39),   w = sum_j w_j 256^j  (LW <= 4 digits),
// so  sum_k a w = sum_s 256^s P_s  with  P_s = sum_{i+j=s} sum_k a_ik w_jk.
// Each P_s is an exact int32 (|a_i w_j| <= 2^14, at most 4 pairs per s, K < 32768) and
// accumulates in TMEM.
//
// Tiles are weight-stationary: a tile is GN = 128 weight rows (the MMA's M, one per TMEM lane) by
// GM = 32 activation rows. One tcgen05.mma.kind::i8 per weight digit j and 32-byte K step takes
// the five activation digit planes stacked along N (5 x 32 rows) as the B operand and writes at
// TMEM column offset 32*j, so digit pair (i, j) lands in column block i+j: S = LA+LW-1 blocks of
// 32 columns (<= 256), two accumulators in the 512 TMEM columns. The kernel is persistent: one CTA
// per SM walks the tiles; operands stream by TMA (GK-byte K stages with the matching swizzle, no
// multicast) through a ring of stages while one thread issues the MMAs; the epilogue of one tile (eight warps)
// overlaps the MMAs of the next. In the epilogue each thread owns one weight row n, so a warp's
// stores of an output row are 32 consecutive int64 (coalesced, residual loads likewise).
// The S partials combine in 64-bit arithmetic (sum = 2^32 H + L, H and L below 2^56) into
// lo64(floor(sum * 2^row_shift / 2^shift)) -- bit-identical to the reference's Int128 result.
// Every mbarrier wait is bounded: on timeout the kernel records an error, waits (bounded) for its
// outstanding copies, frees TMEM and returns.
#include <cuda.h>

#include <cstring>

#include "slx_attr.h"
#include "slx_device.cuh"
#include "slx_exact.cuh"
#include "slx_gemm.h"
#include "slx_kernels.h"
#include "tc_ptx.cuh"

namespace slx {
namespace tc {

constexpr int EPI_WARPS = 16;  // four per TMEM lane quarter, each eight of the tile's activation rows
constexpr int THREADS = 32 * (2 + EPI_WARPS);
constexpr int NACC = 2;       // TMEM accumulators (tile parity picks one)

struct Params {
    int M, N, nkb, shift, tiles_n, tiles;  // tiles: weight tiles fastest, so resident CTAs share activation tiles
    int64_t* C;
    int64_t ldc;
    const int64_t* R;
    int64_t ldr;
    const int* skip;  // nonzero: an operand did not fit its digits, the exact kernel runs instead
    int* err;         // set on a bounded-wait timeout
    // the weight row n was stored as w >> row_shift[n] (its common trailing zeros)
    const int8_t* row_shift;
    long long wait_limit;  // SM clock cycles before a wait on the pipeline gives up
    int stall_mma;         // test hook: the MMA warp issues nothing (the pipeline's waits then run out)
    // the exact CUDA-core product the CTAs compute instead when *skip is set (A null: nothing)
    const int64_t* A;
    int64_t lda;
    int K;
    WDesc W;
};

// Bounded spin on an mbarrier phase without suspending (the MMA issuer's waits are short and on the
// critical path): `limit` SM clock cycles, then false.
__device__ __forceinline__ bool mbar_spin(uint32_t bar, uint32_t parity, long long limit) {
    if (mbar_try(bar, parity)) return true;
    const long long t0 = clock64();
    for (;;) {
#pragma unroll 1
        for (int i = 0; i < 64; i++)
            if (mbar_try(bar, parity)) return true;
        if (clock64() - t0 > limit) return false;
    }
}

// The exact fallback out of line, so its Int128 accumulators do not weigh on the register
// allocation of the tensor-core path (the kernel runs one or the other).
__device__ __noinline__ void exact_fallback(const Params& p, int64_t (*xs)[XBM + 1]) {
    exact_gemm_tiles(p.A, p.lda, p.M, p.K, p.W, p.C, p.ldc, p.shift, p.R, p.ldr, xs, xs + XBK, blockIdx.x, gridDim.x);
}

template <int LW>
__host__ __device__ constexpr int gemm_stages() {
    return (int)((227 * 1024 - 2048) / ((size_t)LW * GN * GK + (size_t)LA * GM * GK)) > 6
               ? 6
               : (int)((227 * 1024 - 2048) / ((size_t)LW * GN * GK + (size_t)LA * GM * GK));
}

// Descriptor of a K-major operand staged with the swizzle that matches GK-byte rows.
__device__ __forceinline__ uint64_t kdesc(uint32_t addr) { return GK == 128 ? sw128_desc(addr) : sw64_desc(addr); }

template <int LW>
__global__ void __launch_bounds__(THREADS, 1)
k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW, Params p) {
    constexpr int S = LA + LW - 1;
    constexpr int ACC = S * GM;  // columns per accumulator
    static_assert(NACC * ACC <= 512 && S <= 8, "TMEM holds 512 columns; the epilogue combines at most 8 blocks");
    constexpr int W_ST = LW * GN * GK, A_ST = LA * GM * GK, STAGE = W_ST + A_ST;
    constexpr int nst = gemm_stages<LW>();
    constexpr uint32_t IDESC = idesc_i8(LA * GM);
    extern __shared__ uint8_t smem_raw[];
    if (p.skip && *p.skip) {  // an operand did not fit its digits: the exact product, on CUDA cores
        if (p.A) exact_fallback(p, (int64_t(*)[XBM + 1])smem_raw);
        return;
    }

    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = (uint64_t*)(smem + (size_t)nst * STAGE);
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + nst);
    const uint32_t tfull0 = smem_u32(bars + 2 * nst), tfree0 = smem_u32(bars + 2 * nst + NACC);
    const uint32_t drain = smem_u32(bars + 2 * nst + 2 * NACC);  // MMAs retired, after a failed wait
    uint32_t* tmem_slot = (uint32_t*)(bars + 2 * nst + 2 * NACC + 1);
    const long long lim = p.wait_limit > 0 ? p.wait_limit : kWaitCycles;
    __shared__ int s_fail;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        s_fail = 0;
        for (int i = 0; i < nst; i++) {
            mbar_init(full0 + 8 * i, 1);
            mbar_init(empty0 + 8 * i, 1);
        }
        for (int b = 0; b < NACC; b++) {
            mbar_init(tfull0 + 8 * b, 1);
            mbar_init(tfree0 + 8 * b, EPI_WARPS);
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
    const int q4 = warp & 3, sub = (warp - 2) >> 2;  // epilogue: TMEM lane quarter, eight of the GM rows
    const uint32_t lane_base = (uint32_t)(32 * q4) << 16;
    // Every MMA accumulates (digit pairs of different j share column blocks): start from zero.
    if (warp >= 2) {
#pragma unroll
        for (int b = 0; b < NACC; b++)
#pragma unroll
            for (int s = 0; s < S; s++) tmem_st8_zero(tmem + lane_base + b * ACC + s * GM + 8 * sub);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t sbase = smem_u32(smem);

    if (warp == 0) {
        if (lane == 0) {  // TMA producer, running ahead across tiles
            int g = 0, s = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < p.tiles; t += gridDim.x) {
                const int m0 = (t / p.tiles_n) * GM, n0 = (t % p.tiles_n) * GN;
                for (int kb = 0; kb < p.nkb; kb++, g++) {
                    if (!mbar_wait(empty0 + 8 * s, ph ^ 1u, lim) || *(volatile int*)&s_fail) {
                        s_fail = 1;
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(full0 + 8 * s, STAGE);
                    tma_load_4d(sbase + s * STAGE, &tmW, kb * GK, n0, 0, 0, full0 + 8 * s);
                    tma_load_4d(sbase + s * STAGE + W_ST, &tmA, kb * GK, m0, 0, 0, full0 + 8 * s);
                    if (++s == nst) { s = 0; ph ^= 1u; }
                }
            }
            if (!ok)  // let copies still in flight land before the CTA exits (they always complete)
                for (int j = g - nst < 0 ? 0 : g - nst; j < g; j++) mbar_wait(full0 + 8 * (j % nst), (uint32_t)(j / nst) & 1u);
        }
    } else if (warp == 1) {
        if (lane == 0 && !p.stall_mma) {  // MMA issuer
            int lt = 0, s = 0;
            uint32_t ph = 0;
            bool ok = true, issued = false;
            for (int t = blockIdx.x; ok && t < p.tiles; t += gridDim.x, lt++) {
                const int b = lt & 1;
                if (!mbar_spin(tfree0 + 8 * b, ((uint32_t)(lt >> 1) & 1u) ^ 1u, lim)) { ok = false; break; }
                fence_after();
                const uint32_t d = tmem + b * ACC;
                for (int kb = 0; kb < p.nkb; kb++) {
                    if (!mbar_spin(full0 + 8 * s, ph, lim)) { ok = false; break; }
                    fence_after();
                    const uint32_t w = sbase + s * STAGE, a = w + W_ST;
#pragma unroll
                    for (int kk = 0; kk < GK / 32; kk++) {
                        const uint64_t bdesc = kdesc(a + kk * 32);
#pragma unroll
                        for (int j = 0; j < LW; j++) umma_i8(d + j * GM, kdesc(w + j * (GN * GK) + kk * 32), bdesc, IDESC, 1u);
                    }
                    umma_commit(empty0 + 8 * s);
                    issued = true;
                    if (++s == nst) { s = 0; ph ^= 1u; }
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
    } else {  // epilogue: thread = weight row n (TMEM lane), eight of the tile's activation rows
        int lt = 0;
        for (int t = blockIdx.x; t < p.tiles; t += gridDim.x, lt++) {
            const int b = lt & 1;
            const int m0 = (t / p.tiles_n) * GM, n0 = (t % p.tiles_n) * GN;
            const int n = n0 + 32 * q4 + lane;
            const bool n_ok = n < p.N;
            // out = lo64(floor(sum * 2^rs / 2^shift)), sum = 2^32 H + L, e = shift - rs:
            //   e <= 0: (H << 32-e) + (L << -e);  0 < e <= 32: (H << 32-e) + (L >> e);
            //   e > 32: (H + (L >> 32)) >> (e - 32).
            const int e = p.shift - ((p.row_shift && n_ok) ? p.row_shift[n] : 0);
            const bool ok = __all_sync(0xffffffffu, mbar_wait(tfull0 + 8 * b, (uint32_t)(lt >> 1) & 1u, lim));
            if (!ok) { s_fail = 1; break; }
            fence_after();
            const uint32_t ta = tmem + lane_base + b * ACC + 8 * sub;
            {
                constexpr int c = 0;
                uint32_t v[S][8];
#pragma unroll
                for (int s = 0; s < S; s++) tmem_ld8(ta + s * GM + c, v[s]);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int s = 0; s < S; s++) tmem_st8_zero(ta + s * GM + c);
                int64_t out[8];
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    uint64_t L = 0, H = 0;
#pragma unroll
                    for (int s = 0; s < S && s < 4; s++) L += (uint64_t)(int64_t)(int32_t)v[s][j] << (8 * s);
#pragma unroll
                    for (int s = 4; s < S; s++) H += (uint64_t)(int64_t)(int32_t)v[s][j] << (8 * (s - 4));
                    uint64_t o;
                    if (e <= 0) {
                        o = (-e >= 64 ? 0 : L << -e) + (32 - e >= 64 ? 0 : H << (32 - e));
                    } else if (e <= 32) {
                        o = (H << (32 - e)) + (uint64_t)((int64_t)L >> e);
                    } else {
                        const int64_t q = (int64_t)H + ((int64_t)L >> 32);
                        o = (uint64_t)(e - 32 >= 64 ? (q >> 63) : q >> (e - 32));
                    }
                    out[j] = (int64_t)o;
                }
                const int mb = m0 + 8 * sub + c;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const int m = mb + j;
                    if (n_ok && m < p.M) {
                        int64_t o = out[j];
                        if (p.R) o = wadd(o, p.R[(int64_t)m * p.ldr + n]);
                        p.C[(int64_t)m * p.ldc + n] = o;
                    }
                }
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
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

// Same digits, four consecutive elements a thread: two 16-byte loads, one 32-bit store per plane
// (rows of A 16-byte aligned, K a multiple of 4).
__global__ void k_split_a4(const int64_t* __restrict__ A, int64_t lda, int M, int K, int Mpad, int Kpad,
                           int8_t* __restrict__ planes, int* overflow) {
    const int quads = Kpad / 4;
    const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (idx >= (int64_t)Mpad * quads) return;
    const int row = (int)(idx / quads), k0 = (int)(idx % quads) * 4;
    int64_t x[4] = {0, 0, 0, 0};
    if (row < M && k0 < K) {
        const longlong2 lo = *(const longlong2*)(A + (int64_t)row * lda + k0);
        const longlong2 hi = *(const longlong2*)(A + (int64_t)row * lda + k0 + 2);
        x[0] = lo.x; x[1] = lo.y; x[2] = hi.x; x[3] = hi.y;
    }
    static_assert(LA == 5, "digit_words4 forms five digits");
    uint32_t pk[LA];
    bool bad = false;
    digit_words4(x[0], x[1], x[2], x[3], pk, bad);
    if (bad) atomicOr(overflow, 1);
#pragma unroll
    for (int i = 0; i < LA; i++) *(uint32_t*)(planes + ((int64_t)i * Mpad + row) * Kpad + k0) = pk[i];
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
    bool bad = false;
    int64_t x[16];
#pragma unroll
    for (int j = 0; j < 16; j++) x[j] = (t < T && k0 + j < hd) ? X[(b * T + t) * ld + (int64_t)h * hd + k0 + j] : 0;
#pragma unroll
    for (int q = 0; q < 4; q++) {
        uint32_t w[LA];
        digit_words4(x[4 * q], x[4 * q + 1], x[4 * q + 2], x[4 * q + 3], w, bad);
#pragma unroll
        for (int i = 0; i < LA; i++) pk[i][q] = w[i];
    }
    if (bad) atomicOr(overflow, 1);
#pragma unroll
    for (int i = 0; i < LA; i++)
        *(uint4*)(planes + ((bh * LA + i) * tpad + t) * kpad + k0) = make_uint4(pk[i][0], pk[i][1], pk[i][2], pk[i][3]);
}

// ApplyRoPE (Math/IntegerAttention.cs:35-58) fused with the head digit split: X row (b*T + t), head h,
// values rotated in place as the reference does (pairs p, p + hd/2 at position t, Int128 products
// >> 30), and their balanced digits written to planes[(b*nh + h)][i][t][k] as k_split_heads does
// (t < tpad, k < kpad, zero padded). A thread owns four pairs of a head row (positions 4q..4q+3 and
// their partners half + 4q..): it rewrites them, writes both digit quads, and zeroes its share of
// the row's padding columns hd..kpad. Rows t >= T get zero digits. hd is a power of two >= 16.
// Without WB the rotated values go to the digit planes only (the int64 rows keep their unrotated
// values; the exact attention, when it runs, rotates them itself first).
// One launch serves q and k: threads [0, a.total) take the head rows of a, the rest those of b.
struct RopeHeads {
    int64_t* X;
    int64_t ld;
    int nh, tpad;
    int8_t* planes;
    int64_t total;  // threads: B * nh * tpad * hd / 8
};
template <bool WB>
__global__ void __launch_bounds__(256, 6) k_rope_split_heads(RopeHeads ja, RopeHeads jb, int T, int hd, int kpad,
                                                             const int64_t* __restrict__ cs,
                                                             const int64_t* __restrict__ sn, int* overflow) {
    int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const bool second = idx >= ja.total;
    if (second) idx -= ja.total;
    if (idx >= (second ? jb.total : ja.total)) return;
    int64_t* const X = second ? jb.X : ja.X;
    const int64_t ld = second ? jb.ld : ja.ld;
    const int nh = second ? jb.nh : ja.nh, tpad = second ? jb.tpad : ja.tpad;
    int8_t* const planes = second ? jb.planes : ja.planes;
    const int half = hd / 2, qpr = half / 4;  // threads per head row
    const int q = (int)(idx % qpr);
    const int64_t r = idx / qpr;  // over (b*nh + h) * tpad + t
    const int t = (int)(r % tpad);
    const int64_t bh = r / tpad;
    const int h = (int)(bh % nh);
    const int64_t b = bh / nh;
    const int p0 = 4 * q;
    int64_t ya[4] = {0, 0, 0, 0}, yb[4] = {0, 0, 0, 0};  // rotated values at p0.. and half + p0..
    bool bad = false;
    if (t < T) {
        int64_t* row = X + (b * T + t) * ld + (int64_t)h * hd;
        const longlong2 a0 = *(const longlong2*)(row + p0), a1 = *(const longlong2*)(row + p0 + 2);
        const longlong2 b0 = *(const longlong2*)(row + half + p0), b1 = *(const longlong2*)(row + half + p0 + 2);
        const int64_t xa[4] = {a0.x, a0.y, a1.x, a1.y}, xb[4] = {b0.x, b0.y, b1.x, b1.y};
        const int64_t* crow = cs + (int64_t)t * half + p0;
        const int64_t* srow = sn + (int64_t)t * half + p0;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int64_t c = crow[j], s = srow[j];
            ya[j] = lo64(sar128((i128)((u128)((i128)xa[j] * c) - (u128)((i128)xb[j] * s)), 30));
            yb[j] = lo64(sar128((i128)((u128)((i128)xa[j] * s) + (u128)((i128)xb[j] * c)), 30));
        }
        if (WB) {
            *(longlong2*)(row + p0) = make_longlong2(ya[0], ya[1]);
            *(longlong2*)(row + p0 + 2) = make_longlong2(ya[2], ya[3]);
            *(longlong2*)(row + half + p0) = make_longlong2(yb[0], yb[1]);
            *(longlong2*)(row + half + p0 + 2) = make_longlong2(yb[2], yb[3]);
        }
    }
    uint32_t wa[LA], wb[LA];
    digit_words4(ya[0], ya[1], ya[2], ya[3], wa, bad);
    digit_words4(yb[0], yb[1], yb[2], yb[3], wb, bad);
    const int pad = (kpad - hd) / qpr;  // padding bytes of this thread per plane row (a multiple of 8)
#pragma unroll
    for (int i = 0; i < LA; i++) {
        int8_t* prow = planes + ((bh * LA + i) * tpad + t) * kpad;
        *(uint32_t*)(prow + p0) = wa[i];
        *(uint32_t*)(prow + half + p0) = wb[i];
        for (int z = 0; z < pad; z += 8) *(uint64_t*)(prow + hd + q * pad + z) = 0;
    }
    if (bad) atomicOr(overflow, 1);
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
    // The driver entry point is the same for every device; looked up once (thread-safe static init).
    static const EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return (EncodeTiledFn)p;
        return (EncodeTiledFn) nullptr;
    }();
    return fn;
}

template <int LW>
constexpr size_t stage_bytes() { return (size_t)LW * GN * GK + (size_t)LA * GM * GK; }


int sm_count() { return slx::device_sm_count(); }

template <int LW>
void launch_lw(const CUtensorMap& ta, const CUtensorMap& tw, Params p, cudaStream_t st) {
    constexpr int nst = gemm_stages<LW>();
    const size_t smem = nst * stage_bytes<LW>() + 1024 + (2 * nst + 2 * NACC + 2) * 8;
    slx::ensure_smem((const void*)k_gemm_tc<LW>, smem);
    const int grid = p.tiles < sm_count() ? p.tiles : sm_count();
    k_gemm_tc<LW><<<grid, THREADS, smem, st>>>(ta, tw, p);
}

Params base_params() {
    Params p;
    memset(&p, 0, sizeof p);
    return p;
}
}  // namespace

bool encode_planes(void* map128, void* base, int64_t kpad, int64_t rows, int planes, int box_rows, int64_t batch, int box_k) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || (box_k != 128 && box_k != 64) || kpad % box_k || planes < 1 || planes > 255 || box_rows < 1 ||
        box_rows > 256 || batch < 1)
        return false;
    if (((uintptr_t)base & 15) != 0) return false;
    cuuint64_t dims[4] = {(cuuint64_t)kpad, (cuuint64_t)rows, (cuuint64_t)planes, (cuuint64_t)batch};
    cuuint64_t strides[3] = {(cuuint64_t)kpad, (cuuint64_t)(kpad * rows), (cuuint64_t)(kpad * rows * planes)};
    cuuint32_t box[4] = {(cuuint32_t)box_k, (cuuint32_t)box_rows, (cuuint32_t)planes, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn((CUtensorMap*)map128, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, base, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, box_k == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
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
    if (K % 4 == 0 && lda % 2 == 0 && ((uintptr_t)a & 15) == 0) {
        const int64_t quads = mpad * (kpad / 4);
        k_split_a4<<<(unsigned)((quads + 255) / 256), 256, 0, st>>>(a, lda, M, K, (int)mpad, (int)kpad, planes, overflow);
        return;
    }
    const int64_t chunks = mpad * (kpad / 16);
    k_split_a<<<(unsigned)((chunks + 255) / 256), 256, 0, st>>>(a, lda, M, K, (int)mpad, (int)kpad, planes, overflow);
}

void launch(const void* tmap_a, const void* tmap_w, int lw, int M, int N, int K, int64_t mpad, int64_t npad, int64_t kpad,
            int shift, int64_t* c, int64_t ldc, const int64_t* r, int64_t ldr, const int* skip, int* err, cudaStream_t st,
            const int8_t* row_shift, const WaitOptions* wait, const int64_t* a, int64_t lda, const WDesc* w) {
    Params p = base_params();
    if (a && w) {
        p.A = a; p.lda = lda; p.K = K; p.W = *w;
    }
    p.M = M; p.N = N; p.nkb = (int)(kpad / GK); p.shift = shift;
    p.tiles_n = (int)((npad + GN - 1) / GN);
    // activation tiles up to M only: the digit planes' padding rows (up to the 128-row multiple)
    // hold zeros whose outputs are never stored
    p.tiles = (int)std::min<int64_t>(mpad / GM, (M + GM - 1) / GM) * p.tiles_n;
    p.C = c; p.ldc = ldc; p.R = r; p.ldr = ldr; p.skip = skip; p.err = err; p.row_shift = row_shift;
    if (wait) { p.wait_limit = wait->limit_cycles; p.stall_mma = wait->stall_mma; }
    const CUtensorMap& ta = *(const CUtensorMap*)tmap_a;
    const CUtensorMap& tw = *(const CUtensorMap*)tmap_w;
    switch (lw) {
        case 1: launch_lw<1>(ta, tw, p, st); break;
        case 2: launch_lw<2>(ta, tw, p, st); break;
        case 3: launch_lw<3>(ta, tw, p, st); break;
        default: launch_lw<4>(ta, tw, p, st); break;
    }
}

void rope_split_heads(int64_t* q, int64_t ldq, int nh, int64_t tq, int8_t* qplanes, int64_t* k, int64_t ldk, int nkv,
                      int64_t tk, int8_t* kplanes, int B, int T, int hd, int64_t kpad, const int64_t* cs,
                      const int64_t* sn, int* overflow, cudaStream_t st, bool write_back) {
    const RopeHeads ja{q, ldq, nh, (int)tq, qplanes, (int64_t)B * nh * tq * (hd / 8)};
    const RopeHeads jb{k, ldk, nkv, (int)tk, kplanes, (int64_t)B * nkv * tk * (hd / 8)};
    const int64_t total = ja.total + jb.total;
    if (total <= 0) return;
    const unsigned grid = (unsigned)((total + 255) / 256);
    if (write_back)
        k_rope_split_heads<true><<<grid, 256, 0, st>>>(ja, jb, T, hd, (int)kpad, cs, sn, overflow);
    else
        k_rope_split_heads<false><<<grid, 256, 0, st>>>(ja, jb, T, hd, (int)kpad, cs, sn, overflow);
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
