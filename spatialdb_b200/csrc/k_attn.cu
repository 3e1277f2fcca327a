// k_attn.cu -- exact integer attention: tcgen05 scores, fixed-point softmax and per-term P.V.
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
// k_softmax_pv: e = FixedExp(score - max) (the reference's Taylor recurrence, ten terms suffice
// for 0 <= r < ln 2), p = (e << 30) / sum. With v = v_hi 2^30 + v_lo (0 <= v_lo < 2^30) and
// 0 <= p <= 2^30,
//   floor(p v / 2^30) = p v_hi + floor(p v_lo / 2^30),
// the first part summed in fp64 (exact: sum_s p_s <= 2^30 and |v_hi| < 2^22 keep every partial
// sum an integer below 2^52) and the second as one mad.hi.u32 per term (the sum stays below
// sum_s p_s <= 2^30, so 32 bits hold it). Any row outside these fast ranges (q/k wider than five
// digits, a score difference that wraps, |v_hi| >= 2^22) raises the call's flag, and the exact
// kernel redoes the call.
#include <cuda.h>

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
constexpr int NBUF = 3;                 // TMEM accumulators
constexpr int BUF_COLS = NSH * NK;      // 144
constexpr int EPI = 16;                 // epilogue warps (four per TMEM lane quarter)
constexpr int CW = NK / (EPI / 4);      // key columns of a tile per epilogue warp
constexpr int S_THREADS = 32 * (2 + EPI);
constexpr uint32_t QPLANE = QM * BK;    // one query digit plane, one 128-byte K block
constexpr uint32_t KPLANE = NK * BK;
constexpr uint32_t IDESC_S = idesc_i8(LA * NK);
static_assert(NBUF * BUF_COLS <= 512, "TMEM holds 512 columns");

struct ScoreParams {
    int T, SR, nh, zgroup, nkv, ksteps, shift, mask_mode, window, ntiles, stages;  // SR: score row stride (even)
    int64_t div;
    int dshift;  // log2(div) when div is a power of two, else -1
    int64_t* S;
    int64_t* rmax;
    const int* skip;
    int* err;
};

template <int KB>
__global__ void __launch_bounds__(S_THREADS, 1)
k_scores(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK, ScoreParams p) {
    constexpr uint32_t QBYTES = KB * LA * QPLANE;
    constexpr uint32_t KSTAGE = KB * LA * KPLANE;
    if (*p.skip) return;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int nst = p.stages;
    uint64_t* bars = (uint64_t*)(smem + QBYTES + (size_t)nst * KSTAGE);
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + nst), qfull = smem_u32(bars + 2 * nst);
    const uint32_t done0 = smem_u32(bars + 2 * nst + 1), tfree0 = smem_u32(bars + 2 * nst + 1 + NBUF);
    uint32_t* tmem_slot = (uint32_t*)(bars + 2 * nst + 1 + 2 * NBUF);
    __shared__ int s_fail;
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
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot)));
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

    const int m0 = blockIdx.x * QM, z = blockIdx.y;
    const int zb = (z / p.nh) * p.nkv + (z % p.nh) / p.zgroup;
    const uint32_t sq = smem_u32(smem), sk = sq + QBYTES;

    if (warp == 0) {
        if (lane == 0) {  // TMA producer: the query tile once, then the key tiles through the ring
            mbar_expect_tx(qfull, QBYTES);
#pragma unroll
            for (int kb = 0; kb < KB; kb++) tma_load_4d(sq + kb * LA * QPLANE, &tmQ, kb * BK, m0, 0, z, qfull);
            int issued = 0;
            for (int t = 0; t < p.ntiles; t++) {
                const int s = t % nst;
                if (!mbar_wait(empty0 + 8 * s, ((uint32_t)(t / nst) & 1u) ^ 1u)) { s_fail = 1; break; }
                if (*(volatile int*)&s_fail) break;
                mbar_expect_tx(full0 + 8 * s, KSTAGE);
#pragma unroll
                for (int kb = 0; kb < KB; kb++)
                    tma_load_4d(sk + s * KSTAGE + kb * LA * KPLANE, &tmK, kb * BK, t * NK, 0, zb, full0 + 8 * s);
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
            for (int t = 0; ok && t < p.ntiles; t++) {
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
        for (int t = 0; t < p.ntiles; t++) {
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
            const int n0 = t * NK + CW * part;
            int64_t o[CW];
#pragma unroll
            for (int j = 0; j < CW; j++) {
                const uint64_t L = (uint64_t)(int64_t)(int32_t)v[0][j] + ((uint64_t)(int64_t)(int32_t)v[1][j] << 8) +
                                   ((uint64_t)(int64_t)(int32_t)v[2][j] << 16) + ((uint64_t)(int64_t)(int32_t)v[3][j] << 24);
                const uint64_t H = (uint64_t)(int64_t)(int32_t)v[4][j] + ((uint64_t)(int64_t)(int32_t)v[5][j] << 8) +
                                   ((uint64_t)(int64_t)(int32_t)v[6][j] << 16) + ((uint64_t)(int64_t)(int32_t)v[7][j] << 24) +
                                   ((uint64_t)(int64_t)(int32_t)v[8][j] << 32);
                int64_t x = (int64_t)((H << (32 - p.shift)) + (uint64_t)((int64_t)L >> p.shift));
                const int n = n0 + j;
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
        if (part == 0 && row_ok) {
#pragma unroll
            for (int i = 1; i < EPI / 4; i++) mx = max(mx, s_max[i][32 * q4 + lane]);
            p.rmax[(int64_t)z * p.T + row] = mx;
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

template <int KB>
constexpr int score_stages() { return KB == 1 ? 6 : 2; }

template <int KB>
constexpr size_t score_smem() {
    return (size_t)KB * LA * QPLANE + (size_t)score_stages<KB>() * KB * LA * KPLANE + 1024 +
           (2 * score_stages<KB>() + 1 + 2 * NBUF + 1) * 8;
}

template <int KB>
void launch_scores_kb(const CUtensorMap& tq, const CUtensorMap& tk, ScoreParams p, dim3 grid, cudaStream_t st) {
    p.stages = score_stages<KB>();
    constexpr size_t smem = score_smem<KB>();
    static_assert(smem <= 227 * 1024, "score kernel shared memory");
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(k_scores<KB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        configured = true;
    }
    k_scores<KB><<<grid, S_THREADS, smem, st>>>(tq, tk, p);
}

// ---------------------------------------------------------------------------------------------
// softmax, then P.V
// ---------------------------------------------------------------------------------------------
// FixedExp(x) for the softmax's x = score - max (IntegerTranscendentals.cs FixedExp): k = -ceil(-x / ln2),
// r = x - k ln2 in [0, ln2), e^r by the truncating Taylor recurrence (exp_taylor30), then e^r >> -k.
// x > 0 (a wrapped difference) and x near long.MinValue (where the reference's own range reduction
// wraps) set bad.
SLX_DEV uint32_t exp_nonpos30(int64_t x, bool& bad) {
    constexpr int64_t LN2 = 744261117;  // (long)(0.6931471805599453 * 2^30)
    if (x > 0 || x < -(1LL << 62)) { bad = true; return 0; }
    if (x < -30 * LN2) return 0;  // a shift of 31 or more clears e^r < 2^31
    const int64_t nx = -x;        // < 2^35, exact in double
    int64_t c = (int64_t)((double)nx * (1.0 / (double)LN2));
    int64_t r = c * LN2 - nx;     // c = ceil(nx / ln2) <=> 0 <= r < ln2
    if (r < 0) { c++; r += LN2; }
    else if (r >= LN2) { c--; r -= LN2; }
    return exp_taylor30((uint32_t)r) >> c;  // c <= 30
}

// floor(e * 2^30 / sum) for e <= 2^30 and sum in [1, 2^41): an fp64 estimate (within one) corrected
// by the exact remainder.
SLX_DEV uint32_t p_div(uint32_t e, uint64_t sum, double inv30) {
    int64_t q = (int64_t)((double)e * inv30);
    int64_t r = (int64_t)(((uint64_t)e << 30) - (uint64_t)q * sum);
    if (r < 0) q--;
    else if (r >= (int64_t)sum) q++;
    return (uint32_t)q;
}

SLX_DEV void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
SLX_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
SLX_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

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

// V -> v >> 30 as fp64 ([T][HD]), 4 * (v mod 2^30) as uint32 ([T][HD], each P.V thread's four columns
// 2g, 2g+1, HD/2+2g, HD/2+2g+1 adjacent) and, for the tensor-core P.V, the two balanced base-256 digits
// of v >> 30 as key-major int8 planes [2][HD][Tpad] (keys past T zero), per (sequence, kv head).
// |v >> 30| >= 2^22 sets the flag (the fp64 sums would not be exact); v >> 30 outside two digits sets
// pvsel (the fp64 P.V runs instead of the tensor-core one).
constexpr int SV_KEYS = 64;  // keys per k_split_v block

template <int HD>
__global__ __launch_bounds__(256) void k_split_v(const int64_t* __restrict__ V, int64_t ldv, int T, int Tpad, int nkv,
                                                 double* __restrict__ Vh, uint32_t* __restrict__ Vl,
                                                 int8_t* __restrict__ Vd, const int* __restrict__ skip, int* flag,
                                                 int* pvsel) {
    __shared__ int16_t s_hi[HD][SV_KEYS + 2];  // v >> 30 of the tile's keys (two-digit values; others flagged)
    if (*skip) return;
    const int zk = blockIdx.y, b = zk / nkv, kvh = zk % nkv, k0 = blockIdx.x * SV_KEYS;
    const int64_t base = (int64_t)zk * T * HD;
    bool bad = false, wide = false;
    for (int i = threadIdx.x; i < SV_KEYS * HD; i += 256) {  // key-major: coalesced along the head's columns
        const int sl = i / HD, d = i % HD, s = k0 + sl;
        int64_t hi = 0;
        if (s < T) {
            const int64_t v = V[((int64_t)b * T + s) * ldv + (int64_t)kvh * HD + d];
            hi = v >> 30;
            bad |= hi < -(1LL << 22) || hi >= (1LL << 22);
            wide |= hi < -32640 || hi > 32639;
            Vh[base + (int64_t)s * HD + d] = (double)hi;
            const int g = d < HD / 2 ? d >> 1 : (d - HD / 2) >> 1, j = d < HD / 2 ? (d & 1) : 2 + (d & 1);
            Vl[base + (int64_t)s * HD + 4 * g + j] = (uint32_t)(v & ((1LL << 30) - 1)) << 2;
        }
        s_hi[d][sl] = (int16_t)(hi < -32640 || hi > 32639 ? 0 : hi);
    }
    if (bad) atomicOr(flag, 1);
    if (wide) atomicOr(pvsel, 1);
    __syncthreads();
    int8_t* vd = Vd + (int64_t)zk * 2 * HD * Tpad + k0;
    for (int i = threadIdx.x; i < HD * SV_KEYS; i += 256) {  // column-major: each plane row's keys contiguous
        const int d = i / SV_KEYS, sl = i % SV_KEYS;
        const int hi = s_hi[d][sl];
        const int d0 = ((hi + 128) & 255) - 128, d1 = (hi - d0) >> 8;
        vd[(int64_t)d * Tpad + sl] = (int8_t)d0;
        vd[((int64_t)HD + d) * Tpad + sl] = (int8_t)d1;
    }
}

// ---- P.V on CUDA cores with fp64 high parts (any head size; the tensor-core kernel's fallback)
constexpr int PR = 32;  // query rows per block

template <int HD>
struct Pv {
    static constexpr int CPT = 4;                      // columns per thread: 2c, 2c+1, HD/2+2c, HD/2+2c+1
    static constexpr int RPT = HD >= 64 ? 4 : HD / 16; // rows per thread
    static constexpr int CG = HD / CPT, RG = PR / RPT;
    static constexpr int THREADS = CG * RG;            // 128 (hd <= 64), 256 (128), 512 (256)
    static constexpr int VT = HD >= 256 ? 8 : 16;      // keys per chunk
    static constexpr int PUS = VT + 4;                 // p row strides (4-word bank offset per row)
    static constexpr int PDS = VT + 2;
    static constexpr int MINB = THREADS <= 128 ? 4 : 1;
    // one staging buffer: v >> 30 (fp64), 4 (v mod 2^30) (uint32), p (uint32)
    static constexpr int VH_BYTES = VT * HD * 8, VL_BYTES = VT * HD * 4, PU_BYTES = PR * PUS * 4;
    static constexpr int BUF = VH_BYTES + VL_BYTES + PU_BYTES;
    static constexpr size_t SMEM = 2 * (size_t)BUF + (size_t)PR * PDS * 8;
};

// PR query rows of one head over chunks of VT keys: p, v >> 30 and 4 (v mod 2^30) arrive by cp.async
// into one of two buffers while the other chunk computes; p is widened to fp64 once per chunk.
// Thread (rg, cg) owns rows rg*RPT .. and columns 2cg, 2cg+1, HD/2+2cg, HD/2+2cg+1. With run_if,
// runs only when *run_if is set.
template <int HD>
__global__ __launch_bounds__(Pv<HD>::THREADS, Pv<HD>::MINB) void k_pv_fp64(
    const int64_t* S, int SR, const double* __restrict__ Vh, const uint32_t* __restrict__ Vl, int64_t* __restrict__ O,
    int64_t ldo, int T, int nh, int nkv, const int* __restrict__ skip, const int* __restrict__ run_if) {
    using C = Pv<HD>;
    constexpr int TH = C::THREADS, VT = C::VT, RPT = C::RPT, CG = C::CG, PUS = C::PUS, PDS = C::PDS;
    if (*skip || (run_if && !*run_if)) return;
    extern __shared__ __align__(16) uint8_t sm[];
    double* Pd = (double*)(sm + 2 * C::BUF);  // [PR][PDS]
    const int h = blockIdx.y, b = blockIdx.z, t0 = blockIdx.x * PR;
    const int z = b * nh + h, zk = b * nkv + h / (nh / nkv);
    const int T4 = (T + 3) & ~3;
    const int cg = threadIdx.x % CG, rg = threadIdx.x / CG;
    const int c0 = 2 * cg, c1 = HD / 2 + 2 * cg;
    const double* vh0 = Vh + (int64_t)zk * T * HD;
    const uint32_t* vl0 = Vl + (int64_t)zk * T * HD;
    const uint32_t sbase = tc::smem_u32(sm);
    auto issue = [&](int k0, int buf) {
        const uint32_t dst = sbase + buf * C::BUF;
        const int keys = min(VT, T - k0);
        for (int g = threadIdx.x; g < C::VH_BYTES / 16; g += TH) {  // v >> 30: HD/2 granules a key
            const int s = g / (HD / 2);
            cp_async16(dst + g * 16, s < keys ? vh0 + (int64_t)k0 * HD + g * 2 : vh0, s < keys ? 16u : 0u);
        }
        for (int g = threadIdx.x; g < C::VL_BYTES / 16; g += TH) {  // 4 (v mod 2^30): HD/4 granules a key
            const int s = g / (HD / 4);
            cp_async16(dst + C::VH_BYTES + g * 16, s < keys ? vl0 + (int64_t)k0 * HD + g * 4 : vl0, s < keys ? 16u : 0u);
        }
        for (int g = threadIdx.x; g < PR * (VT / 4); g += TH) {  // p: VT/4 granules a row
            const int r = g / (VT / 4), s = k0 + 4 * (g % (VT / 4));
            const int t = t0 + r;
            const bool ok = t < T && s < T4;
            const uint32_t* src = ok ? (const uint32_t*)(S + ((int64_t)z * T + t) * SR) + s : (const uint32_t*)S;
            cp_async16(dst + C::VH_BYTES + C::VL_BYTES + (r * PUS + 4 * (g % (VT / 4))) * 4, src, ok ? 16u : 0u);
        }
        cp_async_commit();
    };
    double ah[RPT][4];
    uint32_t al[RPT][4];
#pragma unroll
    for (int r = 0; r < RPT; r++)
#pragma unroll
        for (int c = 0; c < 4; c++) { ah[r][c] = 0.0; al[r][c] = 0; }
    issue(0, 0);
    for (int k0 = 0, buf = 0; k0 < T; k0 += VT, buf ^= 1) {
        cp_async_wait_all();
        __syncthreads();  // chunk k0 is in for every thread; the other buffer and Pd are free
        if (k0 + VT < T) issue(k0 + VT, buf ^ 1);
        const double* Vhs = (const double*)(sm + buf * C::BUF);
        const uint32_t* Vls = (const uint32_t*)(sm + buf * C::BUF + C::VH_BYTES);
        const uint32_t* Pu = (const uint32_t*)(sm + buf * C::BUF + C::VH_BYTES + C::VL_BYTES);
        for (int i = threadIdx.x; i < PR * VT; i += TH) {
            const int r = i / VT, s = i % VT;
            Pd[r * PDS + s] = (double)Pu[r * PUS + s];
        }
        __syncthreads();
#pragma unroll 2
        for (int s = 0; s < VT; s += 4) {
            uint4 pu[RPT];
#pragma unroll
            for (int r = 0; r < RPT; r++) pu[r] = *(const uint4*)(Pu + (rg * RPT + r) * PUS + s);
#pragma unroll
            for (int u = 0; u < 4; u += 2) {
                const double2 ha0 = *(const double2*)(Vhs + (s + u) * HD + c0);
                const double2 ha1 = *(const double2*)(Vhs + (s + u) * HD + c1);
                const double2 hb0 = *(const double2*)(Vhs + (s + u + 1) * HD + c0);
                const double2 hb1 = *(const double2*)(Vhs + (s + u + 1) * HD + c1);
                const uint4 la = *(const uint4*)(Vls + (s + u) * HD + 4 * cg);
                const uint4 lb = *(const uint4*)(Vls + (s + u + 1) * HD + 4 * cg);
#pragma unroll
                for (int r = 0; r < RPT; r++) {
                    const double2 pd = *(const double2*)(Pd + (rg * RPT + r) * PDS + s + u);
                    const uint32_t pa = u == 0 ? pu[r].x : pu[r].z, pb = u == 0 ? pu[r].y : pu[r].w;
                    ah[r][0] = fma(pd.y, hb0.x, fma(pd.x, ha0.x, ah[r][0]));
                    ah[r][1] = fma(pd.y, hb0.y, fma(pd.x, ha0.y, ah[r][1]));
                    ah[r][2] = fma(pd.y, hb1.x, fma(pd.x, ha1.x, ah[r][2]));
                    ah[r][3] = fma(pd.y, hb1.y, fma(pd.x, ha1.y, ah[r][3]));
                    al[r][0] += __umulhi(pa, la.x) + __umulhi(pb, lb.x);
                    al[r][1] += __umulhi(pa, la.y) + __umulhi(pb, lb.y);
                    al[r][2] += __umulhi(pa, la.z) + __umulhi(pb, lb.z);
                    al[r][3] += __umulhi(pa, la.w) + __umulhi(pb, lb.w);
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < RPT; r++) {
        const int t = t0 + rg * RPT + r;
        if (t >= T) continue;
        int64_t* orow = O + ((int64_t)b * T + t) * ldo + (int64_t)h * HD;
        orow[c0] = __double2ll_rz(ah[r][0]) + (int64_t)al[r][0];
        orow[c0 + 1] = __double2ll_rz(ah[r][1]) + (int64_t)al[r][1];
        orow[c1] = __double2ll_rz(ah[r][2]) + (int64_t)al[r][2];
        orow[c1 + 1] = __double2ll_rz(ah[r][3]) + (int64_t)al[r][3];
    }
}

// ---- P.V with the linear part on the tensor cores (head sizes 16, 32, 64)
//   sum_s floor(p v / 2^30) = sum_s p v_hi + sum_s floor(p v_lo / 2^30).
// sum_s p v_hi is a GEMM: p (<= 2^30) as four balanced base-256 digits is the A operand (128 query
// rows, built by the CUDA cores into a 64-byte-swizzled tile per 64-key chunk), v_hi as two digits
// stacked along N (2 x HD rows, key-major planes from k_split_v) the B operand; digit pair (i, j)
// accumulates in TMEM column block i+j (5 blocks of HD int32 columns, each below 2^31 for T < 2^16).
// The CUDA cores add floor(p v_lo / 2^30) = umulhi(p, 4 v_lo) per term, as in k_pv_fp64.
constexpr int PM = 128;  // query rows per block (MMA M)
constexpr int PVT = 64;  // keys per chunk: two 32-key MMA K steps

template <int HD>
struct PvTc {
    static constexpr int TH = 512;                       // compute threads; one more warp issues the MMAs
    static constexpr int CG = HD / 4, RG = TH / CG, RPT = PM / RG;  // thread (rg, cg): rows rg + RG*r
    static constexpr int NB = 2 * HD;                    // B rows: v digit j, column c at j*HD + c
    static constexpr int NS = 5;                         // column blocks
    static constexpr int COLS = NS * HD;
    static constexpr int ALLOC = COLS <= 64 ? 64 : COLS <= 128 ? 128 : COLS <= 256 ? 256 : 512;
    static constexpr int PUS = PVT + 4;                  // p row stride (uint32), rows 4 banks apart
    static constexpr int PD_B = 4 * PM * 64;             // p digits [4][PM][64 B], 64-byte swizzle
    static constexpr int VD_B = NB * 64;                 // v digits [NB][64 B], 64-byte swizzle
    static constexpr int PU_B = PM * PUS * 4, VL_B = PVT * HD * 4;
    static constexpr int BUF = (PD_B + VD_B + PU_B + VL_B + 1023) / 1024 * 1024;
    static constexpr int FSL = HD + 1;                   // floor-sum tile row stride (uint32)
    static constexpr int EQ = HD / 8 < 4 ? HD / 8 : 4;   // epilogue warps per TMEM lane quarter (8 columns each step)
    static constexpr size_t SMEM = 2 * (size_t)BUF + 1024 + 64;
    static_assert(PM * FSL * 4 <= PU_B, "floor sums reuse a p buffer");
};

SLX_DEV uint32_t sw64_off(int row, int g) { return (uint32_t)(row * 64 + ((g ^ ((row >> 1) & 3)) << 4)); }

template <int HD>
__global__ void __launch_bounds__(PvTc<HD>::TH + 32, 1)
k_pv_tc(const int64_t* S, int SR, const int8_t* __restrict__ Vd, int Tpad, const uint32_t* __restrict__ Vl,
        int64_t* __restrict__ O, int64_t ldo, int T, int nh, int nkv, const int* __restrict__ skip,
        const int* __restrict__ pvsel, int* err) {
    using C = PvTc<HD>;
    constexpr int TH = C::TH, RPT = C::RPT, CG = C::CG, RG = C::RG, PUS = C::PUS;
    constexpr uint32_t IDESC = idesc_u8s8(C::NB);  // p's digits are its bytes (0 <= p <= 2^30)
    if (*skip || *pvsel) return;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = (uint64_t*)(sm + 2 * C::BUF);
    const uint32_t done0 = smem_u32(bars), accd = smem_u32(bars + 2);
    uint32_t* tmem_slot = (uint32_t*)(bars + 3);
    __shared__ int s_fail;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.y, b = blockIdx.z, t0 = blockIdx.x * PM;
    const int z = b * nh + h, zk = b * nkv + h / (nh / nkv);
    const int T4 = (T + 3) & ~3;
    const int nch = (T + PVT - 1) / PVT;
    if (threadIdx.x == 0) {
        s_fail = 0;
        mbar_init(done0, 1);
        mbar_init(done0 + 8, 1);
        mbar_init(accd, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == TH / 32) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "n"(C::ALLOC));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    if (warp < TH / 32) {  // every MMA accumulates: start from zero
        const uint32_t lb = (uint32_t)(32 * (warp & 3)) << 16;
        for (int c = 8 * (warp >> 2); c < C::COLS; c += 8 * (TH / 128)) tmem_st8_zero(tmem + lb + c);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    fence_before();
    __syncthreads();
    fence_after();

    const uint32_t sbase = smem_u32(sm);
    const int8_t* vd0 = Vd + (int64_t)zk * C::NB * Tpad;
    const uint32_t* vl0 = Vl + (int64_t)zk * T * HD;
    // chunk k0's p rows, 4 (v mod 2^30) and v digits into buffer buf (all compute threads)
    auto issue = [&](int k0, int buf) {
        const uint32_t dst = sbase + buf * C::BUF;
        for (int g = threadIdx.x; g < PM * (PVT / 4); g += TH) {  // p: 16 granules a row
            const int r = g / (PVT / 4), s = k0 + 4 * (g % (PVT / 4));
            const int t = t0 + r;
            const bool ok = t < T && s < T4;
            const uint32_t* src = ok ? (const uint32_t*)(S + ((int64_t)z * T + t) * SR) + s : (const uint32_t*)S;
            cp_async16(dst + C::PD_B + C::VD_B + (r * PUS + 4 * (g % (PVT / 4))) * 4, src, ok ? 16u : 0u);
        }
        const int keys = min(PVT, T - k0);
        for (int g = threadIdx.x; g < C::VL_B / 16; g += TH) {  // 4 (v mod 2^30): HD/4 granules a key
            const int s = g / (HD / 4);
            cp_async16(dst + C::PD_B + C::VD_B + C::PU_B + g * 16, s < keys ? vl0 + (int64_t)k0 * HD + g * 4 : vl0,
                       s < keys ? 16u : 0u);
        }
        for (int g = threadIdx.x; g < C::NB * 4; g += TH) {  // v digits: four 16-byte granules a row
            const int r = g >> 2, q = g & 3;
            cp_async16(dst + C::PD_B + sw64_off(r, q), vd0 + (int64_t)r * Tpad + k0 + 16 * q, 16u);
        }
        cp_async_commit();
    };

    const int cg = threadIdx.x % CG, rg = threadIdx.x / CG;
    const int c0 = 2 * cg, c1 = HD / 2 + 2 * cg;
    uint32_t al[RPT][4];
#pragma unroll
    for (int r = 0; r < RPT; r++)
#pragma unroll
        for (int c = 0; c < 4; c++) al[r][c] = 0;
    if (warp < TH / 32) issue(0, 0);
    for (int c = 0; c < nch; c++) {
        const int buf = c & 1, k0 = c * PVT;
        uint8_t* bp = sm + buf * C::BUF;
        const uint32_t* Pu = (const uint32_t*)(bp + C::PD_B + C::VD_B);
        const uint32_t* Vls = (const uint32_t*)(bp + C::PD_B + C::VD_B + C::PU_B);
        if (warp < TH / 32) cp_async_wait_all();
        __syncthreads();  // chunk c is in; every thread finished chunk c-1's CUDA-core part
        if (warp < TH / 32) {
            if (c + 1 < nch) {
                // the other buffer's digit tiles were read by chunk c-1's MMAs
                if (c >= 1 && !mbar_wait(done0 + 8 * (buf ^ 1), (uint32_t)((c - 1) >> 1) & 1u)) s_fail = 1;
                issue(k0 + PVT, buf ^ 1);
            }
            // p digits of chunk c: (row, 16-key granule) items. 0 <= p <= 2^30, so its unsigned
            // base-256 digits are its four bytes (the MMA reads A as u8); a 4 x 4 byte transpose per
            // 4 keys puts byte i of keys k..k+3 into plane i
            for (int it = threadIdx.x; it < PM * 4; it += TH) {
                const int r = it >> 2, q = it & 3;
                uint32_t pk[4][4];
#pragma unroll
                for (int w4 = 0; w4 < 4; w4++) {
                    const uint4 pv = *(const uint4*)(Pu + r * PUS + 16 * q + 4 * w4);
                    const uint32_t ab_lo = __byte_perm(pv.x, pv.y, 0x5140), ab_hi = __byte_perm(pv.x, pv.y, 0x7362);
                    const uint32_t cd_lo = __byte_perm(pv.z, pv.w, 0x5140), cd_hi = __byte_perm(pv.z, pv.w, 0x7362);
                    pk[0][w4] = __byte_perm(ab_lo, cd_lo, 0x5410);
                    pk[1][w4] = __byte_perm(ab_lo, cd_lo, 0x7632);
                    pk[2][w4] = __byte_perm(ab_hi, cd_hi, 0x5410);
                    pk[3][w4] = __byte_perm(ab_hi, cd_hi, 0x7632);
                }
#pragma unroll
                for (int i = 0; i < 4; i++)
                    *(uint4*)(bp + i * (PM * 64) + sw64_off(r, q)) = make_uint4(pk[i][0], pk[i][1], pk[i][2], pk[i][3]);
            }
            fence_proxy_async();  // generic-proxy tile writes (and the landed copies) visible to the MMA
        }
        __syncthreads();  // chunk c's digit tiles complete
        if (warp == TH / 32) {
            if (lane == 0) {
                fence_after();
                const uint32_t pd = sbase + buf * C::BUF, vd = pd + C::PD_B;
#pragma unroll
                for (int kk = 0; kk < PVT / 32; kk++) {
                    const uint64_t bdesc = tc::sw64_desc(vd + kk * 32);
#pragma unroll
                    for (int i = 0; i < 4; i++)
                        umma_i8(tmem + i * HD, tc::sw64_desc(pd + i * (PM * 64) + kk * 32), bdesc, IDESC, 1u);
                }
                umma_commit(done0 + 8 * buf);
                if (c == nch - 1) umma_commit(accd);
            }
        } else {
            // floor(p v_lo / 2^30) on the CUDA cores
#pragma unroll 2
            for (int s = 0; s < PVT; s += 4) {
                uint4 pu[RPT];
#pragma unroll
                for (int r = 0; r < RPT; r++) pu[r] = *(const uint4*)(Pu + (rg + RG * r) * PUS + s);
#pragma unroll
                for (int u = 0; u < 4; u += 2) {
                    const uint4 la = *(const uint4*)(Vls + (s + u) * HD + 4 * cg);
                    const uint4 lb = *(const uint4*)(Vls + (s + u + 1) * HD + 4 * cg);
#pragma unroll
                    for (int r = 0; r < RPT; r++) {
                        const uint32_t pa = u == 0 ? pu[r].x : pu[r].z, pb = u == 0 ? pu[r].y : pu[r].w;
                        al[r][0] += __umulhi(pa, la.x) + __umulhi(pb, lb.x);
                        al[r][1] += __umulhi(pa, la.y) + __umulhi(pb, lb.y);
                        al[r][2] += __umulhi(pa, la.z) + __umulhi(pb, lb.z);
                        al[r][3] += __umulhi(pa, la.w) + __umulhi(pb, lb.w);
                    }
                }
            }
        }
    }
    __syncthreads();  // every chunk's CUDA-core part is done: buffer 0's p region takes the floor sums
    uint32_t* fs = (uint32_t*)(sm + C::PD_B + C::VD_B);
    if (warp < TH / 32) {
#pragma unroll
        for (int r = 0; r < RPT; r++) {
            const int row = rg + RG * r;
            fs[row * C::FSL + c0] = al[r][0];
            fs[row * C::FSL + c0 + 1] = al[r][1];
            fs[row * C::FSL + c1] = al[r][2];
            fs[row * C::FSL + c1 + 1] = al[r][3];
        }
    }
    __syncthreads();
    if (warp < 4 * C::EQ) {
        const bool ok = __all_sync(0xffffffffu, mbar_wait(accd, 0));
        if (!ok) s_fail = 1;
        fence_after();
        const int q4 = warp & 3, part = warp >> 2;
        const int row = 32 * q4 + lane, t = t0 + row;
        const uint32_t ta = tmem + ((uint32_t)(32 * q4) << 16);
        int64_t* orow = O + ((int64_t)b * T + (t < T ? t : 0)) * ldo + (int64_t)h * HD;
        if (ok) {
#pragma unroll 1
            for (int cc = 8 * part; cc < HD; cc += 8 * C::EQ) {
                uint32_t v[C::NS][8];
#pragma unroll
                for (int s2 = 0; s2 < C::NS; s2++) tmem_ld8(ta + s2 * HD + cc, v[s2]);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (t < T) {
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        uint64_t sum = 0;  // sum_s p v_hi = sum of 2^(8 s) P_s, below 2^46 in magnitude
#pragma unroll
                        for (int s2 = 0; s2 < C::NS; s2++) sum += (uint64_t)(int64_t)(int32_t)v[s2][j] << (8 * s2);
                        orow[cc + j] = (int64_t)(sum + fs[row * C::FSL + cc + j]);
                    }
                }
            }
        }
    }
    fence_before();
    __syncthreads();
    if (s_fail && threadIdx.x == 0 && err) atomicOr(err, KERR_TIMEOUT);
    if (warp == TH / 32) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(C::ALLOC));
    }
}

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

template <int HD>
void launch_pv(int B, int T, int nh, int nkv, int64_t* scores, int sr, const int64_t* v, int64_t ldv, double* vh,
               uint32_t* vl, int8_t* vd, int tpad, int64_t* out, int64_t ldo, int* flag, int* pvsel, int* err,
               cudaStream_t st) {
    const dim3 vgrid((unsigned)(tpad / SV_KEYS), (unsigned)(B * nkv));
    k_split_v<HD><<<vgrid, 256, 0, st>>>(v, ldv, T, tpad, nkv, vh, vl, vd, flag, flag, pvsel);
    constexpr bool tcpath = HD <= 64;
    if constexpr (tcpath) {
        // a TMEM column block sums at most two (p byte, v digit) products of 255 * 128 per key:
        // int32 holds them for T < 32896; longer rows take the fp64 P.V
        if (T > 32768) {
            cudaMemsetAsync(pvsel, 1, sizeof(int), st);
            goto fp64;
        }
        constexpr size_t smem = PvTc<HD>::SMEM;
        static_assert(smem <= 227 * 1024, "tensor-core P.V shared memory");
        static bool configured = false;
        if (!configured) {
            cudaFuncSetAttribute(k_pv_tc<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            configured = true;
        }
        dim3 grid((unsigned)((T + PM - 1) / PM), (unsigned)nh, (unsigned)B);
        k_pv_tc<HD><<<grid, PvTc<HD>::TH + 32, smem, st>>>(scores, sr, vd, tpad, vl, out, ldo, T, nh, nkv, flag, pvsel, err);
    }
fp64:
    constexpr size_t smem = Pv<HD>::SMEM;
    static_assert(smem <= 200 * 1024, "P.V shared memory");
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(k_pv_fp64<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        configured = true;
    }
    dim3 grid((unsigned)((T + PR - 1) / PR), (unsigned)nh, (unsigned)B);
    k_pv_fp64<HD><<<grid, Pv<HD>::THREADS, smem, st>>>(scores, sr, vh, vl, out, ldo, T, nh, nkv, flag,
                                                      tcpath ? pvsel : nullptr);
}

struct Layout {
    int64_t kpad, tq, tk, sr, tpad, qbytes, kbytes, sbytes, mbytes, vhbytes, vlbytes, vdbytes;
};

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
    l.vhbytes = round_up((int64_t)B * nkv * T * hd * 8, 256);
    l.vlbytes = round_up((int64_t)B * nkv * T * hd * 4, 256);
    l.tpad = round_up(T, PVT);
    l.vdbytes = (int64_t)B * nkv * 2 * hd * l.tpad;
    return l;
}
}  // namespace

size_t attention_tc_workspace(int B, int T, int nh, int nkv, int hd) {
    const Layout l = layout(B, T, nh, nkv, hd);
    return (size_t)(256 + l.qbytes + l.kbytes + l.sbytes + l.mbytes + l.vhbytes + l.vlbytes + l.vdbytes);
}

bool attention_tc_supported(int T, int nh, int nkv, int hd) {
    const bool hd_ok = hd == 16 || hd == 32 || hd == 64 || hd == 128 || hd == 256;
    return hd_ok && T > 0 && nkv > 0 && nh % nkv == 0;
}

int attention_tc(const int64_t* q, int64_t ldq, const int64_t* k, int64_t ldk, const int64_t* v, int64_t ldv,
                 int64_t* out, int64_t ldo, int B, int T, int nh, int nkv, int hd, int score_shift, int64_t sqrt_hd,
                 int mode, int window, void* ws, int* err, cudaStream_t st) {
    if (score_shift < 0 || score_shift > 32 || sqrt_hd < 1) return -1;
    const Layout l = layout(B, T, nh, nkv, hd);
    uint8_t* base = (uint8_t*)ws;
    int* flag = (int*)base;
    int8_t* qp = (int8_t*)(base + 256);
    int8_t* kp = qp + l.qbytes;
    int64_t* scores = (int64_t*)(kp + l.kbytes);
    int64_t* rmax = (int64_t*)((uint8_t*)scores + l.sbytes);
    double* vh = (double*)((uint8_t*)rmax + l.mbytes);
    uint32_t* vl = (uint32_t*)((uint8_t*)vh + l.vhbytes);
    int8_t* vd = (int8_t*)((uint8_t*)vl + l.vlbytes);
    int* pvsel = flag + 1;  // v >> 30 beyond two digits: the fp64 P.V instead of the tensor-core one
    alignas(64) unsigned char mq[128], mk[128];
    if (!encode_planes(mq, qp, l.kpad, l.tq, LA, QM, (int64_t)B * nh) ||
        !encode_planes(mk, kp, l.kpad, l.tk, LA, NK, (int64_t)B * nkv))
        return -1;
    cudaMemsetAsync(flag, 0, 2 * sizeof(int), st);
    split_heads(q, ldq, B, T, nh, hd, l.tq, l.kpad, qp, flag, st);
    split_heads(k, ldk, B, T, nkv, hd, l.tk, l.kpad, kp, flag, st);

    ScoreParams sp;
    sp.T = T; sp.SR = (int)l.sr; sp.nh = nh; sp.zgroup = nh / nkv; sp.nkv = nkv;
    sp.ksteps = (hd + 31) / 32;
    sp.shift = score_shift; sp.mask_mode = mode; sp.window = window;
    sp.ntiles = (int)(l.tk / NK);
    sp.stages = 0;
    sp.div = sqrt_hd;
    sp.dshift = (sqrt_hd & (sqrt_hd - 1)) == 0 ? __builtin_ctzll((unsigned long long)sqrt_hd) : -1;
    sp.S = scores; sp.rmax = rmax; sp.skip = flag; sp.err = err;
    const dim3 sgrid((unsigned)(l.tq / QM), (unsigned)(B * nh));
    if (l.kpad == BK) launch_scores_kb<1>(*(const CUtensorMap*)mq, *(const CUtensorMap*)mk, sp, sgrid, st);
    else launch_scores_kb<2>(*(const CUtensorMap*)mq, *(const CUtensorMap*)mk, sp, sgrid, st);

    const int64_t rows = (int64_t)B * nh * T;
    k_softmax<<<(unsigned)((rows + SM_ROWS - 1) / SM_ROWS), 32 * SM_ROWS, 0, st>>>(scores, (int)l.sr, rmax, T, (int)rows,
                                                                                  flag, flag);
    const int tp = (int)l.tpad, sr = (int)l.sr;
    switch (hd) {
        case 16: launch_pv<16>(B, T, nh, nkv, scores, sr, v, ldv, vh, vl, vd, tp, out, ldo, flag, pvsel, err, st); break;
        case 32: launch_pv<32>(B, T, nh, nkv, scores, sr, v, ldv, vh, vl, vd, tp, out, ldo, flag, pvsel, err, st); break;
        case 64: launch_pv<64>(B, T, nh, nkv, scores, sr, v, ldv, vh, vl, vd, tp, out, ldo, flag, pvsel, err, st); break;
        case 128: launch_pv<128>(B, T, nh, nkv, scores, sr, v, ldv, vh, vl, vd, tp, out, ldo, flag, pvsel, err, st); break;
        default: launch_pv<256>(B, T, nh, nkv, scores, sr, v, ldv, vh, vl, vd, tp, out, ldo, flag, pvsel, err, st); break;
    }
    // the exact kernel redoes the whole call when anything fell outside the fast ranges
    attention(q, ldq, k, ldk, v, ldv, out, ldo, B, T, nh, nkv, hd, score_shift, sqrt_hd, mode, window, st, flag);
    return hd <= 64 ? 8 : 7;
}

}  // namespace slx
