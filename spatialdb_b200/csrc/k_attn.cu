// k_attn.cu -- exact integer attention: tcgen05 scores, fixed-point softmax and a directed-rounding fp64 P.V.
//
// Reference semantics (Math/IntegerAttention.cs:60-109, 165-202, 246-289, 333-377), per head:
//   score[t][s] = (long)((sum_d q[t][d]*k[s][d]) >> shift) / ISqrt64(hd)   (masked slots: -2^29)
//   p[t][s]     = FixedSoftmax(score[t][:])                                 (IntegerTranscendentals.cs:71-97)
//   out[t][d]   = sum_s (long)(((Int128)p[t][s] * v[s][d]) >> 30)          (floor per term, long sum)
//
// k_scores: q and k of a head are split into 5 balanced base-256 digits (k_split_heads). One CTA
// keeps its 128-query tile's digit planes in shared memory and streams 16-key tiles of k by TMA;
// per 32-wide K step one tcgen05.mma per query digit i multiplies against all five key digits
// stacked along N, so digit pair (i, j) lands in TMEM column block i+j (9 blocks of 16 columns,
// each an exact int32 sum). Three TMEM accumulators rotate so the epilogue of one tile overlaps
// the MMAs of the next. With P_s the block sums (|P_s| < 2^25 for hd <= 256),
//   L = P_0 + 2^8 P_1 + 2^16 P_2 + 2^24 P_3,   H = P_4 + ... + 2^32 P_8,   sum = 2^32 H + L,
// and for 0 <= shift <= 32, floor(sum / 2^shift) = 2^(32-shift) H + (L >> shift) in wrapping
// 64-bit arithmetic -- the reference's (long)(Int128 >> shift) without 128-bit work. The epilogue
// also keeps each row's maximum for the softmax.
//
// k_softmax: e = FixedExp(score - max) (the reference's Taylor recurrence, ten terms suffice for
// 0 <= r < ln 2), p = (e << 30) / sum, so 0 <= p <= 2^30 and sum_s p_s <= 2^30.
//
// k_pv: floor(p v / 2^30) per term, summed, as one fp64 FMA rounded toward minus infinity into an
// accumulator kept in [2^52, 2^53) (the window where the doubles are the integers): exact for
// |v| < 2^50, which keeps every partial sum inside the window. Any row outside the fast ranges (q/k
// wider than five digits, a score difference that wraps, |v| >= 2^50) raises the call's flag, and
// the exact kernel redoes the call.
#include <cuda.h>

#include <algorithm>

#include "slx_attr.h"
#include "slx_device.cuh"
#include "slx_gemm.h"
#include "slx_kernels.h"
#include "tc_ptx.cuh"

namespace slx {
namespace {

using namespace tc;

// ---------------------------------------------------------------------------------------------
// scores
// ---------------------------------------------------------------------------------------------
constexpr int QM = 128;                 // query rows per CTA (TMEM lanes)
constexpr int NK = 16;                  // keys per tile
constexpr int NSH = 2 * LA - 1;         // shift blocks of 16 columns
// TMEM accumulators per CTA: with a query tile of one 128-byte K block (hd <= 128) two CTAs share
// an SM, each with one accumulator in 256 columns, and one CTA's epilogue overlaps the other's MMAs
// (measured faster than one CTA with three accumulators); wider heads keep one CTA with three.
template <int KB> __host__ __device__ constexpr int nbuf() { return KB == 1 ? 1 : 3; }
template <int KB> __host__ __device__ constexpr int score_ctas() { return KB == 1 ? 2 : 1; }
constexpr int NBUF_MAX = 3;
constexpr int BUF_COLS = NSH * NK;      // 144
constexpr int EPI = 16;                 // epilogue warps (four per TMEM lane quarter)
constexpr int CW = NK / (EPI / 4);      // key columns of a tile per epilogue warp
constexpr int S_THREADS = 32 * (2 + EPI);
constexpr uint32_t QPLANE = QM * BK;    // one query digit plane, one 128-byte K block
constexpr uint32_t KPLANE = NK * BK;
constexpr uint32_t IDESC_S = idesc_i8(LA * NK);
static_assert(NBUF_MAX * BUF_COLS <= 512 && BUF_COLS <= 256, "TMEM holds 512 columns");

// Work split of a score launch: units (query tile rt, head z) numbered u = z * ntr + rt; the first
// `whole` run over every key tile; when the units do not fill the last wave of resident CTAs, each of
// the remaining ones is split into S key ranges, whose parts write their own scores and a partial row
// maximum, and the last part of a unit to finish (an atomic count) writes the unit's row maxima.
struct ScorePlan {
    int ntr = 0, units = 0, whole = 0, rem = 0, S = 1;
    int blocks() const { return whole + rem * S; }
    size_t partial_bytes() const { return S > 1 ? (size_t)rem * S * QM * 8 : 0; }
};

struct ScoreParams {
    int T, SR, nh, zgroup, nkv, ksteps, shift, mask_mode, window, ntiles, stages;  // SR: score row stride (even)
    ScorePlan plan;
    int* cnt;        // per split unit, zeroed before the launch
    int64_t* pmax;   // [rem][S][QM] partial row maxima
    int64_t div;
    int dshift;  // log2(div) when div is a power of two, else -1
    int64_t* S;
    int64_t* rmax;
    const int* skip;
    int* err;
};

// FAST: shift 30, a power-of-two divisor and no mask (the encoders' attention): constant shifts and
// no per-score mask tests.
template <int KB, bool FAST>
__global__ void __launch_bounds__(S_THREADS, score_ctas<KB>())
k_scores(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK, ScoreParams p) {
    constexpr uint32_t QBYTES = KB * LA * QPLANE;
    constexpr uint32_t KSTAGE = KB * LA * KPLANE;
    constexpr int NBUF = nbuf<KB>();
    constexpr uint32_t TCOLS = score_ctas<KB>() == 2 ? 256 : 512;
    if (*p.skip) return;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int nst = p.stages;
    uint64_t* bars = (uint64_t*)(smem + QBYTES + (size_t)nst * KSTAGE);
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + nst), qfull = smem_u32(bars + 2 * nst);
    const uint32_t done0 = smem_u32(bars + 2 * nst + 1), tfree0 = smem_u32(bars + 2 * nst + 1 + NBUF);
    uint32_t* tmem_slot = (uint32_t*)(bars + 2 * nst + 1 + 2 * NBUF);
    __shared__ int s_fail, s_last;
    __shared__ int64_t s_max[EPI / 4][QM];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        s_fail = 0;
        for (int i = 0; i < nst; i++) {
            mbar_init(full0 + 8 * i, 1);
            mbar_init(empty0 + 8 * i, 1);
        }
        mbar_init(qfull, 1);
        for (int b = 0; b < NBUF; b++) {
            mbar_init(done0 + 8 * b, 1);
            mbar_init(tfree0 + 8 * b, EPI);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "n"(TCOLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    const int q4 = warp & 3, part = (warp - 2) >> 2;           // epilogue: lane quarter, column part
    const uint32_t lane_base = (uint32_t)(32 * q4) << 16;
    if (warp >= 2) {  // every MMA accumulates: start from zero
#pragma unroll 1
        for (int b = 0; b < NBUF; b++)
#pragma unroll
            for (int s = 0; s < NSH; s++) tmem_st4_zero(tmem + lane_base + b * BUF_COLS + s * NK + CW * part);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    fence_before();
    __syncthreads();
    fence_after();

    const int item = blockIdx.x;
    int u = item, pid = 0, t_lo = 0, t_hi = p.ntiles;
    if (item >= p.plan.whole) {  // part pid of split unit (item - whole) / S: key tiles [t_lo, t_hi)
        pid = (item - p.plan.whole) % p.plan.S;
        u = p.plan.whole + (item - p.plan.whole) / p.plan.S;
        t_lo = pid * p.ntiles / p.plan.S;
        t_hi = (pid + 1) * p.ntiles / p.plan.S;
    }
    const int nloc = t_hi - t_lo;
    const int m0 = (u % p.plan.ntr) * QM, z = u / p.plan.ntr;
    const int zb = (z / p.nh) * p.nkv + (z % p.nh) / p.zgroup;
    const uint32_t sq = smem_u32(smem), sk = sq + QBYTES;

    if (warp == 0) {
        if (lane == 0) {  // TMA producer: the query tile once, then the key tiles through the ring
            mbar_expect_tx(qfull, QBYTES);
#pragma unroll
            for (int kb = 0; kb < KB; kb++) tma_load_4d(sq + kb * LA * QPLANE, &tmQ, kb * BK, m0, 0, z, qfull);
            int issued = 0;
            for (int t = 0; t < nloc; t++) {  // t: the CTA's own tile count, t_lo + t the key tile
                const int s = t % nst;
                if (!mbar_wait(empty0 + 8 * s, ((uint32_t)(t / nst) & 1u) ^ 1u)) { s_fail = 1; break; }
                if (*(volatile int*)&s_fail) break;
                mbar_expect_tx(full0 + 8 * s, KSTAGE);
#pragma unroll
                for (int kb = 0; kb < KB; kb++)
                    tma_load_4d(sk + s * KSTAGE + kb * LA * KPLANE, &tmK, kb * BK, (t_lo + t) * NK, 0, zb, full0 + 8 * s);
                issued = t + 1;
            }
            if (*(volatile int*)&s_fail) {  // let copies still in flight land before the CTA exits
                mbar_wait(qfull, 0);
                for (int t = issued - nst < 0 ? 0 : issued - nst; t < issued; t++)
                    mbar_wait(full0 + 8 * (t % nst), (uint32_t)(t / nst) & 1u);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            bool ok = mbar_wait(qfull, 0);
            for (int t = 0; ok && t < nloc; t++) {
                const int s = t % nst, b = t % NBUF;
                if (!mbar_wait(full0 + 8 * s, (uint32_t)(t / nst) & 1u) ||
                    !mbar_wait(tfree0 + 8 * b, ((uint32_t)(t / NBUF) & 1u) ^ 1u)) {
                    ok = false;
                    break;
                }
                fence_after();
                const uint32_t kst = sk + s * KSTAGE, d = tmem + b * BUF_COLS;
                for (int kk = 0; kk < p.ksteps; kk++) {
                    const uint32_t koff = (kk >> 2) * (LA * KPLANE) + (kk & 3) * 32;
                    const uint32_t qoff = (kk >> 2) * (LA * QPLANE) + (kk & 3) * 32;
                    const uint64_t bdesc = sw128_desc(kst + koff);
#pragma unroll
                    for (int i = 0; i < LA; i++) umma_i8(d + i * NK, sw128_desc(sq + qoff + i * QPLANE), bdesc, IDESC_S, 1u);
                }
                umma_commit(empty0 + 8 * s);
                umma_commit(done0 + 8 * b);
            }
            if (!ok) s_fail = 1;
        }
    } else {  // epilogue: row = TMEM lane, CW of each tile's 16 keys
        const int row = m0 + 32 * q4 + lane;
        const bool row_ok = row < p.T;
        int64_t* srow = p.S + ((int64_t)z * p.T + (row_ok ? row : 0)) * p.SR;
        const int ws = row - p.window + 1;
        const double rdiv = 1.0 / (double)p.div;
        int64_t mx = INT64_MIN;
#pragma unroll 1
        for (int t = 0; t < nloc; t++) {
            const int b = t % NBUF;
            const bool ok = __all_sync(0xffffffffu, mbar_wait(done0 + 8 * b, (uint32_t)(t / NBUF) & 1u));
            if (!ok) { s_fail = 1; break; }
            fence_after();
            uint32_t v[NSH][CW];
            const uint32_t ta = tmem + lane_base + b * BUF_COLS + CW * part;
#pragma unroll
            for (int s = 0; s < NSH; s++) tmem_ld4(ta + s * NK, v[s]);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
            for (int s = 0; s < NSH; s++) tmem_st4_zero(ta + s * NK);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tfree0 + 8 * b);
            const int n0 = (t_lo + t) * NK + CW * part;
            int64_t o[CW];
#pragma unroll
            for (int j = 0; j < CW; j++) {
                // L and H as sums of int32 x constant products (wide multiply-adds), in wrapping 64 bits
                const int64_t L = (int64_t)(int32_t)v[0][j] + (int64_t)(int32_t)v[1][j] * 256 +
                                  (int64_t)(int32_t)v[2][j] * 65536 + (int64_t)(int32_t)v[3][j] * 16777216;
                const uint64_t H = (uint64_t)((int64_t)(int32_t)v[4][j] + (int64_t)(int32_t)v[5][j] * 256 +
                                              (int64_t)(int32_t)v[6][j] * 65536 + (int64_t)(int32_t)v[7][j] * 16777216) +
                                   ((uint64_t)v[8][j] << 32);
                const int n = n0 + j;
                if (FAST) {
                    int64_t x = (int64_t)((H << 2) + (uint64_t)(L >> 30));
                    x = (int64_t)((uint64_t)x + ((uint64_t)(x >> 63) & (uint64_t)(p.div - 1))) >> p.dshift;  // truncating
                    o[j] = x;
                    if (n < p.T) mx = max(mx, x);
                    continue;
                }
                int64_t x = (int64_t)((H << (32 - p.shift)) + (uint64_t)(L >> p.shift));
                if ((p.mask_mode >= 1 && n > row) || (p.mask_mode == 2 && n < ws)) {
                    x = -(1LL << 29);  // maskValue (IntegerAttention.cs:222)
                } else if (p.dshift >= 0) {  // C# long division truncates toward zero
                    x = (int64_t)((uint64_t)x + ((uint64_t)(x >> 63) & (uint64_t)(p.div - 1))) >> p.dshift;
                } else {
                    x = div_small(x, p.div, rdiv);
                }
                o[j] = x;
                if (n < p.T) mx = max(mx, x);
            }
            if (row_ok) {
                if (n0 + CW <= p.T) {
#pragma unroll
                    for (int j = 0; j < CW; j += 2) *(longlong2*)(srow + n0 + j) = make_longlong2(o[j], o[j + 1]);
                } else {
#pragma unroll
                    for (int j = 0; j < CW; j++)
                        if (n0 + j < p.T) srow[n0 + j] = o[j];
                }
            }
        }
        // row maximum over the column parts
        s_max[part][32 * q4 + lane] = mx;
        asm volatile("bar.sync 1, %0;" ::"n"(32 * EPI) : "memory");
        if (part == 0) {
#pragma unroll
            for (int i = 1; i < EPI / 4; i++) mx = max(mx, s_max[i][32 * q4 + lane]);
            if (item < p.plan.whole) {
                if (row_ok) p.rmax[(int64_t)z * p.T + row] = mx;
            } else {
                p.pmax[(int64_t)(item - p.plan.whole) * QM + 32 * q4 + lane] = mx;
                __threadfence();
            }
        }
    }
    fence_before();
    __syncthreads();
    if (item >= p.plan.whole) {  // the last part of a split unit writes its row maxima
        const int j = (item - p.plan.whole) / p.plan.S;
        if (threadIdx.x == 0) s_last = atomicAdd(p.cnt + j, 1) == p.plan.S - 1;
        __syncthreads();
        if (s_last && threadIdx.x < QM && m0 + (int)threadIdx.x < p.T) {
            __threadfence();
            int64_t mx = INT64_MIN;
            for (int o = 0; o < p.plan.S; o++)
                mx = max(mx, (int64_t)__ldcg((const long long*)p.pmax + ((int64_t)j * p.plan.S + o) * QM + threadIdx.x));
            p.rmax[(int64_t)z * p.T + m0 + threadIdx.x] = mx;
        }
    }
    if (s_fail && threadIdx.x == 0 && p.err) atomicOr(p.err, KERR_TIMEOUT);
    if (warp == 1) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(TCOLS));
    }
}

template <int KB>
constexpr int score_stages() { return 2; }

template <int KB>
constexpr size_t score_smem() {
    return (size_t)KB * LA * QPLANE + (size_t)score_stages<KB>() * KB * LA * KPLANE + 1024 +
           (2 * score_stages<KB>() + 1 + 2 * nbuf<KB>() + 1) * 8;
}

template <int KB>
void launch_scores_kb(const CUtensorMap& tq, const CUtensorMap& tk, ScoreParams p, dim3 grid, cudaStream_t st) {
    p.stages = score_stages<KB>();
    constexpr size_t smem = score_smem<KB>();
    static_assert(smem <= 227 * 1024, "score kernel shared memory");
    static_assert(score_ctas<KB>() == 1 || smem + sizeof(int64_t) * (EPI / 4) * QM + 64 <= 113 * 1024,
                  "two score CTAs per SM");
    if (p.shift == 30 && p.dshift >= 0 && p.mask_mode == 0) {
        slx::ensure_smem((const void*)k_scores<KB, true>, smem);
        k_scores<KB, true><<<grid, S_THREADS, smem, st>>>(tq, tk, p);
    } else {
        slx::ensure_smem((const void*)k_scores<KB, false>, smem);
        k_scores<KB, false><<<grid, S_THREADS, smem, st>>>(tq, tk, p);
    }
}

// ---------------------------------------------------------------------------------------------
// softmax, then P.V
// ---------------------------------------------------------------------------------------------
// FixedExp(x) for the softmax's x = score - max (IntegerTranscendentals.cs FixedExp): k = -ceil(-x / ln2),
// r = x - k ln2 in [0, ln2) (ln2_reduce, on the fp64 pipe), e^r by the truncating Taylor recurrence
// (exp_taylor30_fp), then e^r >> -k. x > 0 (a wrapped difference) and x near long.MinValue (where the
// reference's own range reduction wraps) set bad.
SLX_DEV uint32_t exp_nonpos30(int64_t x, bool& bad) {
    constexpr int64_t LN2 = 744261117;  // (long)(0.6931471805599453 * 2^30)
    if (x > 0 || x < -(1LL << 62)) { bad = true; return 0; }
    if (x < -30 * LN2) return 0;  // a shift of 31 or more clears e^r < 2^31
    double r;
    const int k = ln2_reduce(d_i64(x), r);  // -30 <= k <= 0
    return exp_taylor30_fp((uint32_t)rd_i32(r + RD_BASE), r) >> -k;
}

// floor(e * 2^30 / sum) for e <= 2^30 and sum in [2^30, 2^41) (the softmax's sum includes the
// maximum's own e = 2^30): the fp64 product e * inv30, inv30 = 2^30 / sum rounded to nearest, is
// within 2^-23 of the exact quotient (at most 2^30), so its floor is exact unless the product lies
// within 2^-22 of an integer; only there the exact 64-bit remainder decides.
SLX_DEV uint32_t p_div(uint32_t e, uint64_t sum, double inv30) {
    const double ed = d_u32(e);
    const double y = rd_floor(ed, inv30);  // 1.5 * 2^52 + floor(e * inv30)
    int64_t q = rd_i32(y);
    const double frac = __fma_rn(ed, inv30, -(y - RD_BASE));  // e * inv30 - floor(e * inv30)
    if (frac < 0x1p-22 || frac > 1.0 - 0x1p-22) {
        const int64_t r = (int64_t)(((uint64_t)e << 30) - (uint64_t)q * sum);
        if (r < 0) q--;
        else if (r >= (int64_t)sum) q++;
    }
    return (uint32_t)q;
}

SLX_DEV void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
SLX_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
SLX_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
SLX_DEV void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// FixedSoftmax of score rows in place, one warp per row (row stride SR int64): pass one writes
// e = FixedExp(score - max) as uint32 over the first half of the row's storage (each 256-key chunk is
// read completely before its e values are written), pass two rewrites them as p = (e << 30) / sum
// and zeroes p up to the next multiple of four keys. A row outside the fast ranges sets the flag.
constexpr int SM_ROWS = 8;  // rows (warps) per block
__global__ __launch_bounds__(32 * SM_ROWS) void k_softmax(int64_t* S, int SR, const int64_t* __restrict__ rmax, int T,
                                                          int rows, const int* __restrict__ skip, int* flag) {
    constexpr int SU = 8;  // keys per lane per chunk: loads batched, exps interleaved
    if (*skip) return;
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * SM_ROWS + (threadIdx.x >> 5);  // over z * T + t
    if (row >= rows) return;
    const int T4 = (T + 3) & ~3;
    const int64_t* srow = S + row * SR;
    uint32_t* prow = (uint32_t*)(S + row * SR);
    const int64_t mx = rmax[row];
    uint64_t sum = 0;
    bool bad = false;
    for (int s0 = 0; s0 < T; s0 += 32 * SU) {
        int64_t x[SU];
#pragma unroll
        for (int u = 0; u < SU; u++) {
            const int sk = s0 + 32 * u + lane;
            x[u] = sk < T ? srow[sk] : mx;
        }
        __syncwarp();  // this chunk is read before its e values overwrite the first half of it
#pragma unroll
        for (int u = 0; u < SU; u++) {
            const int sk = s0 + 32 * u + lane;
            const uint32_t e = exp_nonpos30(wsub(x[u], mx), bad);
            if (sk < T) { prow[sk] = e; sum += e; }
        }
    }
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, (unsigned long long)sum, o);
    if (__any_sync(0xffffffffu, bad)) {
        if (lane == 0) atomicOr(flag, 1);
        return;
    }
    __syncwarp();
    if (sum == 0) {  // uniform = one / len
        for (int s = lane; s < T; s += 32) prow[s] = (uint32_t)((1LL << 30) / T);
    } else {
        const double inv30 = 1073741824.0 / (double)sum;
#pragma unroll 4
        for (int s = lane; s < T; s += 32) prow[s] = p_div(prow[s], sum, inv30);
    }
    if (lane < T4 - T) prow[T + lane] = 0;
}

// ---- P.V: one fp64 FMA rounded toward minus infinity per term (any head size)
//   out[t][d] = sum_s floor(p[t][s] v[s][d] / 2^30),   0 <= p <= 2^30,  |v| < 2^50.
// The accumulator starts at 1.5 * 2^52 and holds 1.5 * 2^52 + S with S an integer, |S| < 2^51, so
// every exact value acc + p v / 2^30 lies in [2^52, 2^53), where the doubles are exactly the
// integers: fma_rd(p, v * 2^-30, acc) rounds that value down, which adds floor(p v / 2^30) exactly
// (p and v * 2^-30 are exact doubles and the FMA rounds once). S stays inside the window because
// FixedSoftmax floors every share, so sum_s p_s <= 2^30 and |S| <= max |v| + T. A value with
// |v| >= 2^50 raises the call's flag and the exact kernel redoes the call.
constexpr int PV_TH = 128;  // four warps
constexpr double PV_BASE = 6755399441055744.0;  // 1.5 * 2^52

constexpr int pv_keys_per_chunk(int hd) { return (hd == 256 || hd == 16) ? 8 : 16; }
constexpr int PV_MAX_SPLIT = 1024;  // tail tiles that may be split (counters in the workspace header)

// Work of one P.V launch: tiles of PR query rows of one head, numbered u = (b * nh + h) * ntr + rt.
// The first `whole` tiles run one block each over all keys; when the tiles do not fill the last
// wave of resident blocks (two per SM), the remaining tiles are split into S key ranges each, so
// the tail is S times shorter. A split part writes its exact int64 partial sums to the workspace
// and the last part of a tile to finish (an atomic count per tile) adds them up and writes the
// rows: partial sums of floored terms are integers, so the split changes no bit of the result.
struct PvPlan {
    int ntr = 0, tiles = 0, whole = 0, rem = 0, S = 1;
    // optional: the next projection's activation digit planes ([5][mpad][kpad] int8, row b * T + t,
    // column h * HD + d), written beside the int64 rows; a value needing a sixth digit sets bit 2 of
    // the flag
    int8_t* planes = nullptr;
    int64_t mpad = 0, kpad = 0;
    int blocks() const { return whole + rem * S; }
    size_t partial_bytes() const { return S > 1 ? (size_t)rem * S * 8192 * 8 : 0; }  // PR * HD = 8192
};

PvPlan pv_plan(int hd, int B, int T, int nh) {
    PvPlan pl;
    const int pr = 8192 / hd, vt = pv_keys_per_chunk(hd);
    const int slots = 2 * device_sm_count();
    const int nch = (T + vt - 1) / vt;
    pl.ntr = (T + pr - 1) / pr;
    pl.tiles = pl.ntr * nh * B;
    pl.rem = pl.tiles % slots;
    pl.whole = pl.tiles - pl.rem;
    if (pl.rem == 0 || pl.rem > PV_MAX_SPLIT || nch < 2) {
        pl.whole = pl.tiles;
        pl.rem = 0;
        return pl;
    }
    // tail length in whole-tile times: ceil(rem * S / slots) / S, plus ~3 % for the partials
    double best = 1.0;
    const int smax = std::min(std::min(nch, 16), std::max(1, 3 * slots / pl.rem));
    for (int sp = 2; sp <= smax; sp++) {
        const double tail = (double)((pl.rem * sp + slots - 1) / slots) / sp * 1.03;
        if (tail < 0.95 * best) best = tail, pl.S = sp;
    }
    if (pl.S == 1) pl.whole = pl.tiles, pl.rem = 0;
    return pl;
}

// Register tile of a thread: 8 query rows x 8 columns (64 fp64 accumulators). Per key a thread
// loads its 8 columns of v and its 8 rows of p as four 16-byte shared loads each and issues 64
// DFMAs. Columns of a thread: 2cg, 2cg+1 + 2 CG j (j < 4), so the eight lanes of a quarter warp
// read 128 contiguous bytes of a v row; rows: 8 consecutive, contiguous in the key-major p tile.
//
// Chunks of VT keys move through two raw buffers (int64 v rows and uint32 p granules, filled by
// cp.async) and two converted buffers (v * 2^-30 and p as doubles, p transposed key-major). While
// a block multiplies chunk c out of one converted buffer, its threads convert chunk c + 1 into the
// other, a few values after each key's DFMAs, so the conversions issue beside the fp64 pipe's work
// instead of in a phase of their own; chunk c + 2 is in flight meanwhile.
template <int HD>
struct Pv {
    static constexpr int CG = HD / 8;                    // column groups (lanes per row group)
    static constexpr int RGW = 32 / CG;                  // row groups per warp
    static constexpr int PR = (PV_TH / 32) * RGW * 8;    // query rows per block: 8192 / HD
    static constexpr int VT = pv_keys_per_chunk(HD);     // keys per chunk
    static constexpr int RV = VT * HD * 8;               // raw v: int64 [VT][HD]
    static constexpr int RP = PR * VT * 4;               // raw p: 16-byte granules [VT/4][PR]
    static constexpr int RAW = RV + RP;
    static constexpr int CV = VT * HD * 8;               // converted v: double [VT][HD]
    static constexpr int CONV = CV + VT * PR * 8;        // + converted p: double [VT][PR]
    static constexpr size_t SMEM = 2 * (size_t)RAW + 2 * (size_t)CONV;
    static constexpr int NV = VT * HD / PV_TH;           // v values a thread converts per chunk
    static constexpr int NPG = PR * VT / 4;              // p granules per chunk
    static constexpr int NP = (NPG + PV_TH - 1) / PV_TH; // p granules a thread converts per chunk
    static constexpr int NW = NV + NP;                   // conversion items a thread has per chunk
    static_assert(CG >= 2 && CG <= 32 && RAW % 16 == 0 && CONV % 16 == 0 && VT % 4 == 0, "P.V tiling");
    static_assert(VT * HD % PV_TH == 0, "v conversion");
};

// PR query rows of one head, VT keys at a time (see Pv).
// flag: bit 0 set by the earlier stages (the block returns at once), bit 1 set here when a value
// of v is out of range; either makes the exact kernel redo the call.
template <int HD>
__global__ __launch_bounds__(PV_TH, 2) void k_pv(const int64_t* S, int SR, const int64_t* __restrict__ V,
                                                  int64_t ldv, int64_t* __restrict__ O, int64_t ldo, int T, int nh,
                                                  int nkv, PvPlan pl, int* flag, int* cnt, int64_t* part) {
    using C = Pv<HD>;
    constexpr int VT = C::VT, CG = C::CG, RGW = C::RGW, PR = C::PR;
    if (*flag & 1) return;
    extern __shared__ __align__(16) uint8_t sm[];
    __shared__ int s_last;
    uint8_t* raw_base = sm;                   // raw chunk buffers: [2][RAW]
    uint8_t* conv_base = sm + 2 * C::RAW;     // converted chunk buffers: [2][CONV]
    const int nchunks = (T + VT - 1) / VT;
    const int item = blockIdx.x;
    int u = item, pid = 0, c_lo = 0, c_hi = nchunks;
    if (item >= pl.whole) {  // part pid of split tile (item - whole) / S: chunks [c_lo, c_hi)
        const int j = (item - pl.whole) / pl.S;
        pid = (item - pl.whole) % pl.S;
        u = pl.whole + j;
        c_lo = pid * nchunks / pl.S;
        c_hi = (pid + 1) * nchunks / pl.S;
    }
    const int h = (u / pl.ntr) % nh, b = u / (pl.ntr * nh), t0 = (u % pl.ntr) * PR;
    const int z = b * nh + h, kvh = h / (nh / nkv);
    const int T4 = (T + 3) & ~3;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int cg = lane % CG, r0 = 8 * (warp * RGW + lane / CG);  // first of the thread's 8 rows
    const int64_t* v0 = V + (int64_t)b * T * ldv + (int64_t)kvh * HD;  // key s: v0 + s * ldv
    const uint32_t sbase = tc::smem_u32(sm);
    auto issue = [&](int c, int buf) {
        const int k0 = c * VT;
        const uint32_t dst = sbase + buf * C::RAW;
        const int keys = min(VT, T - k0);
        for (int g = threadIdx.x; g < C::RV / 16; g += PV_TH) {  // v: HD/2 granules a key
            const int s = g / (HD / 2), j = g % (HD / 2);
            cp_async16(dst + g * 16, s < keys ? v0 + (int64_t)(k0 + s) * ldv + 2 * j : v0, s < keys ? 16u : 0u);
        }
        for (int g = threadIdx.x; g < C::NPG; g += PV_TH) {  // p: granule (row r, keys 4q..4q+3) at [q][r]
            const int r = g % PR, q = g / PR, s = k0 + 4 * q;
            const int t = t0 + r;
            const bool ok = t < T && s < T4;
            const uint32_t* src = ok ? (const uint32_t*)(S + ((int64_t)z * T + t) * SR) + s : (const uint32_t*)S;
            cp_async16(dst + C::RV + g * 16, src, ok ? 16u : 0u);
        }
    };
    bool wide = false;
    // item w of a thread's share of converting raw buffer rb into converted buffer cb
    auto convert = [&](int w, int rb, int cb, bool live) {
        const uint8_t* rw = raw_base + rb * C::RAW;
        uint8_t* cv = conv_base + cb * C::CONV;
        if (w < C::NV) {
            const int i = threadIdx.x + w * PV_TH;  // exact for |v| < 2^53
            const int64_t x = ((const int64_t*)rw)[i];
            wide |= live && ((x >> 30) < -(1LL << 20) || (x >> 30) >= (1LL << 20));
            ((double*)cv)[i] = (double)x * 0x1p-30;
        } else {
            const int g = threadIdx.x + (w - C::NV) * PV_TH;
            if (C::NPG % PV_TH == 0 || g < C::NPG) {
                const uint4 u = ((const uint4*)(rw + C::RV))[g];
                const int r = g % PR, q = g / PR;
                double* Pd = (double*)(cv + C::CV);
                Pd[(4 * q + 0) * PR + r] = (double)u.x;
                Pd[(4 * q + 1) * PR + r] = (double)u.y;
                Pd[(4 * q + 2) * PR + r] = (double)u.z;
                Pd[(4 * q + 3) * PR + r] = (double)u.w;
            }
        }
    };
    double acc[8][8];
#pragma unroll
    for (int r = 0; r < 8; r++)
#pragma unroll
        for (int c = 0; c < 8; c++) acc[r][c] = PV_BASE;
    issue(c_lo, 0);
    cp_async_commit();
    if (c_lo + 1 < c_hi) issue(c_lo + 1, 1);
    cp_async_commit();
    cp_async_wait_1();
    __syncthreads();  // the first chunk's raw rows are in for every thread
#pragma unroll
    for (int w = 0; w < C::NW; w++) convert(w, 0, 0, true);
    for (int c = c_lo; c < c_hi; c++) {
        const int cur = (c - c_lo) & 1;
        cp_async_wait_all();
        // chunk c + 1's raw rows and chunk c's converted values are in for every thread; raw
        // buffer cur (chunk c, converted) and converted buffer cur ^ 1 (chunk c - 1) are free
        __syncthreads();
        if (c + 2 < c_hi) issue(c + 2, cur);
        cp_async_commit();
        const double* Vs = (const double*)(conv_base + cur * C::CONV);
        const double* Pd = (const double*)(conv_base + cur * C::CONV + C::CV);
        const bool live = c + 1 < c_hi;  // raw buffer cur ^ 1 holds a real chunk
#pragma unroll
        for (int s = 0; s < VT; s++) {  // one key at a time: every accumulator once per key
            double2 v[4], p[4];
#pragma unroll
            for (int j = 0; j < 4; j++) v[j] = *(const double2*)(Vs + s * HD + 2 * cg + 2 * CG * j);
#pragma unroll
            for (int i = 0; i < 4; i++) p[i] = *(const double2*)(Pd + s * PR + r0 + 2 * i);
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    acc[2 * i][2 * j] = __fma_rd(p[i].x, v[j].x, acc[2 * i][2 * j]);
                    acc[2 * i][2 * j + 1] = __fma_rd(p[i].x, v[j].y, acc[2 * i][2 * j + 1]);
                    acc[2 * i + 1][2 * j] = __fma_rd(p[i].y, v[j].x, acc[2 * i + 1][2 * j]);
                    acc[2 * i + 1][2 * j + 1] = __fma_rd(p[i].y, v[j].y, acc[2 * i + 1][2 * j + 1]);
                }
#pragma unroll
            for (int w = s * C::NW / VT; w < (s + 1) * C::NW / VT; w++) convert(w, cur ^ 1, cur ^ 1, live);
        }
    }
    // a wide v leaves the rows to the exact kernel; the split parts still count in below, so the
    // per-tile counts stay whole
    if (__syncthreads_or(wide) && threadIdx.x == 0) atomicOr(flag, 2);
    int64_t sum[8][8];
#pragma unroll
    for (int r = 0; r < 8; r++)
#pragma unroll
        for (int c = 0; c < 8; c++) sum[r][c] = (int64_t)(acc[r][c] - PV_BASE);
    if (item >= pl.whole) {
        const int j = (item - pl.whole) / pl.S;
        int64_t* mine = part + (int64_t)(item - pl.whole) * PR * HD;  // [PR][HD]
#pragma unroll
        for (int r = 0; r < 8; r++)
#pragma unroll
            for (int q = 0; q < 4; q++)
                *(longlong2*)(mine + (r0 + r) * HD + 2 * cg + 2 * CG * q) = make_longlong2(sum[r][2 * q], sum[r][2 * q + 1]);
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) s_last = atomicAdd(cnt + j, 1) == pl.S - 1;
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        for (int o = 0; o < pl.S; o++) {
            if (o == pid) continue;
            const int64_t* other = part + ((int64_t)j * pl.S + o) * PR * HD;
#pragma unroll
            for (int r = 0; r < 8; r++)
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const longlong2 x = __ldcg((const longlong2*)(other + (r0 + r) * HD + 2 * cg + 2 * CG * q));
                    sum[r][2 * q] += x.x;
                    sum[r][2 * q + 1] += x.y;
                }
        }
    }
#pragma unroll
    for (int r = 0; r < 8; r++) {
        const int t = t0 + r0 + r;
        if (t >= T) continue;
        int64_t* orow = O + ((int64_t)b * T + t) * ldo + (int64_t)h * HD;
#pragma unroll
        for (int q = 0; q < 4; q++)
            *(longlong2*)(orow + 2 * cg + 2 * CG * q) = make_longlong2(sum[r][2 * q], sum[r][2 * q + 1]);
    }
    if (!pl.planes) return;
    // The digit planes through shared memory: the block's [PR][HD] tile (64 KB, the chunk buffers'
    // space, free once every thread is past the key loop), then four consecutive columns a thread, so
    // a warp writes 128 contiguous bytes of a plane row.
    int64_t* tile = (int64_t*)sm;
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 8; r++)
#pragma unroll
        for (int q = 0; q < 4; q++)
            *(longlong2*)(tile + (r0 + r) * HD + 2 * cg + 2 * CG * q) = make_longlong2(sum[r][2 * q], sum[r][2 * q + 1]);
    __syncthreads();
    bool over = false;
    for (int g = threadIdx.x; g < PR * (HD / 4); g += PV_TH) {
        const int r = g / (HD / 4), c = 4 * (g % (HD / 4));
        const int t = t0 + r;
        if (t >= T) continue;
        const longlong2 x01 = *(const longlong2*)(tile + r * HD + c), x23 = *(const longlong2*)(tile + r * HD + c + 2);
        uint32_t wd[5];
        digit_words4(x01.x, x01.y, x23.x, x23.y, wd, over);
        int8_t* prow = pl.planes + ((int64_t)b * T + t) * pl.kpad + (int64_t)h * HD + c;
#pragma unroll
        for (int i = 0; i < 5; i++) *(uint32_t*)(prow + (int64_t)i * pl.mpad * pl.kpad) = wd[i];
    }
    if (over) atomicOr(flag, 4);
}

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

template <int HD>
void launch_pv(int B, int T, int nh, int nkv, const int64_t* scores, int sr, const int64_t* v, int64_t ldv,
               int64_t* out, int64_t ldo, const PvPlan& pl, int* flag, int* cnt, int64_t* part, cudaStream_t st) {
    using C = Pv<HD>;
    static_assert(C::SMEM <= 112 * 1024, "two P.V blocks per SM");
    static_assert(C::SMEM >= (size_t)C::PR * HD * sizeof(int64_t), "the output tile fits the chunk buffers");
    static_assert(C::VT == pv_keys_per_chunk(HD) && C::PR * HD == 8192, "plan and kernel agree");
    if (((uintptr_t)v & 15) != 0 || (ldv & 1) != 0 || ((uintptr_t)out & 15) != 0 || (ldo & 1) != 0) {
        // rows the 16-byte copies and stores cannot address: the exact kernel
        cudaMemsetAsync(flag, 1, sizeof(int), st);
        return;
    }
    slx::ensure_smem((const void*)k_pv<HD>, C::SMEM);
    k_pv<HD><<<(unsigned)pl.blocks(), PV_TH, C::SMEM, st>>>(scores, sr, v, ldv, out, ldo, T, nh, nkv, pl, flag, cnt,
                                                            part);
}

// Workspace: [0, 256) the call's flag; [256, HDR) the split tiles' counters; then the q and k
// digit planes, the scores, the row maxima and the split parts' partial sums.
constexpr int SC_MAX_SPLIT = 1024;  // score units that may be split (their counters follow the P.V's)
constexpr int64_t WS_HDR = 256 + 4 * PV_MAX_SPLIT + 4 * SC_MAX_SPLIT;
struct Layout {
    int64_t kpad, tq, tk, sr, qbytes, kbytes, sbytes, mbytes, pbytes, xbytes;
};

ScorePlan score_plan(int hd, int B, int T, int nh) {
    ScorePlan pl;
    const int slots = (hd <= BK ? score_ctas<1>() : score_ctas<2>()) * device_sm_count();
    const int nt = (int)(round_up(T, NK) / NK);
    pl.ntr = (int)(round_up(T, QM) / QM);
    pl.units = pl.ntr * nh * B;
    pl.rem = pl.units % slots;
    pl.whole = pl.units - pl.rem;
    if (pl.rem == 0 || pl.rem > SC_MAX_SPLIT || nt < 2) {
        pl.whole = pl.units;
        pl.rem = 0;
        return pl;
    }
    // tail length in whole-unit times: ceil(rem * S / slots) / S, plus ~3 % for the partial maxima
    double best = 1.0;
    const int smax = std::min(std::min(nt, 16), std::max(1, 3 * slots / pl.rem));
    for (int sp = 2; sp <= smax; sp++) {
        const double tail = (double)((pl.rem * sp + slots - 1) / slots) / sp * 1.03;
        if (tail < 0.95 * best) best = tail, pl.S = sp;
    }
    if (pl.S == 1) pl.whole = pl.units, pl.rem = 0;
    return pl;
}

Layout layout(int B, int T, int nh, int nkv, int hd) {
    Layout l;
    l.kpad = round_up(hd, BK);
    l.tq = round_up(T, QM);
    l.tk = round_up(T, NK);
    l.qbytes = round_up((int64_t)B * nh * LA * l.tq * l.kpad, 256);
    l.kbytes = round_up((int64_t)B * nkv * LA * l.tk * l.kpad, 256);
    l.sr = round_up(T, 2);
    l.sbytes = round_up((int64_t)B * nh * T * l.sr * 8, 256);
    l.mbytes = round_up((int64_t)B * nh * T * 8, 256);
    l.pbytes = round_up((int64_t)pv_plan(hd, B, T, nh).partial_bytes(), 256);
    l.xbytes = (int64_t)score_plan(hd, B, T, nh).partial_bytes();
    return l;
}
}  // namespace

size_t attention_tc_workspace(int B, int T, int nh, int nkv, int hd) {
    const Layout l = layout(B, T, nh, nkv, hd);
    return (size_t)(WS_HDR + l.qbytes + l.kbytes + l.sbytes + l.mbytes + l.pbytes + l.xbytes);
}

bool attention_tc_supported(int T, int nh, int nkv, int hd) {
    const bool hd_ok = hd == 16 || hd == 32 || hd == 64 || hd == 128 || hd == 256;
    return hd_ok && T > 0 && nkv > 0 && nh % nkv == 0;
}

int attention_tc(const int64_t* q, int64_t ldq, const int64_t* k, int64_t ldk, const int64_t* v, int64_t ldv,
                 int64_t* out, int64_t ldo, int B, int T, int nh, int nkv, int hd, int score_shift, int64_t sqrt_hd,
                 int mode, int window, void* ws, int* err, cudaStream_t st, const int64_t* rope_cs,
                 const int64_t* rope_sn, int8_t* planes, int64_t mpad, int64_t kpad) {
    if (score_shift < 0 || score_shift > 32 || sqrt_hd < 1) return -1;
    const Layout l = layout(B, T, nh, nkv, hd);
    uint8_t* base = (uint8_t*)ws;
    int* flag = (int*)base;
    int* cnt = (int*)(base + 256);
    int8_t* qp = (int8_t*)(base + WS_HDR);
    int8_t* kp = qp + l.qbytes;
    int64_t* scores = (int64_t*)(kp + l.kbytes);
    int64_t* rmax = (int64_t*)((uint8_t*)scores + l.sbytes);
    int64_t* part = (int64_t*)((uint8_t*)rmax + l.mbytes);
    int64_t* pmax = (int64_t*)((uint8_t*)part + l.pbytes);
    int* scnt = cnt + PV_MAX_SPLIT;
    const ScorePlan spl = score_plan(hd, B, T, nh);
    PvPlan pl = pv_plan(hd, B, T, nh);
    if (planes && kpad == (int64_t)nh * hd && mpad >= (int64_t)B * T) {
        pl.planes = planes;
        pl.mpad = mpad;
        pl.kpad = kpad;
    }
    alignas(64) unsigned char mq[128], mk[128];
    if (!encode_planes(mq, qp, l.kpad, l.tq, LA, QM, (int64_t)B * nh) ||
        !encode_planes(mk, kp, l.kpad, l.tk, LA, NK, (int64_t)B * nkv))
        return -1;
    // the flag and the split units' counters (P.V's, then the score kernel's)
    cudaMemsetAsync(flag, 0, 256 + 4 * (size_t)PV_MAX_SPLIT + 4 * (size_t)spl.rem, st);
    if (rope_cs) {  // ApplyRoPE on q and k, fused with their digit split (the planes get the rotated values)
        rope_split_heads(const_cast<int64_t*>(q), ldq, nh, l.tq, qp, const_cast<int64_t*>(k), ldk, nkv, l.tk, kp, B, T, hd,
                         l.kpad, rope_cs, rope_sn, flag, st, false);
    } else {
        split_heads(q, ldq, B, T, nh, hd, l.tq, l.kpad, qp, flag, st);
        split_heads(k, ldk, B, T, nkv, hd, l.tk, l.kpad, kp, flag, st);
    }

    ScoreParams sp;
    sp.T = T; sp.SR = (int)l.sr; sp.nh = nh; sp.zgroup = nh / nkv; sp.nkv = nkv;
    sp.ksteps = (hd + 31) / 32;
    sp.shift = score_shift; sp.mask_mode = mode; sp.window = window;
    sp.ntiles = (int)(l.tk / NK);
    sp.stages = 0;
    sp.div = sqrt_hd;
    sp.dshift = (sqrt_hd & (sqrt_hd - 1)) == 0 ? __builtin_ctzll((unsigned long long)sqrt_hd) : -1;
    sp.S = scores; sp.rmax = rmax; sp.skip = flag; sp.err = err;
    sp.plan = spl;
    sp.cnt = scnt;
    sp.pmax = pmax;
    const dim3 sgrid((unsigned)spl.blocks());
    if (l.kpad == BK) launch_scores_kb<1>(*(const CUtensorMap*)mq, *(const CUtensorMap*)mk, sp, sgrid, st);
    else launch_scores_kb<2>(*(const CUtensorMap*)mq, *(const CUtensorMap*)mk, sp, sgrid, st);

    const int64_t rows = (int64_t)B * nh * T;
    k_softmax<<<(unsigned)((rows + SM_ROWS - 1) / SM_ROWS), 32 * SM_ROWS, 0, st>>>(scores, (int)l.sr, rmax, T, (int)rows,
                                                                                  flag, flag);
    const int sr = (int)l.sr;
    switch (hd) {
        case 16: launch_pv<16>(B, T, nh, nkv, scores, sr, v, ldv, out, ldo, pl, flag, cnt, part, st); break;
        case 32: launch_pv<32>(B, T, nh, nkv, scores, sr, v, ldv, out, ldo, pl, flag, cnt, part, st); break;
        case 64: launch_pv<64>(B, T, nh, nkv, scores, sr, v, ldv, out, ldo, pl, flag, cnt, part, st); break;
        case 128: launch_pv<128>(B, T, nh, nkv, scores, sr, v, ldv, out, ldo, pl, flag, cnt, part, st); break;
        default: launch_pv<256>(B, T, nh, nkv, scores, sr, v, ldv, out, ldo, pl, flag, cnt, part, st); break;
    }
    // the exact kernel redoes the whole call when anything fell outside the fast ranges, on q and k
    // rotated in place first (the fast path rotated only their digit planes)
    int n = rope_cs ? 5 : 6;  // the q and k digit splits (one launch with RoPE), scores, softmax, P.V, exact
    if (rope_cs) {
        n += rope_rows(const_cast<int64_t*>(q), ldq, B, T, nh, hd, rope_cs, rope_sn, st, flag);
        n += rope_rows(const_cast<int64_t*>(k), ldk, B, T, nkv, hd, rope_cs, rope_sn, st, flag);
    }
    attention(q, ldq, k, ldk, v, ldv, out, ldo, B, T, nh, nkv, hd, score_shift, sqrt_hd, mode, window, st, flag);
    return n;
}

}  // namespace slx
