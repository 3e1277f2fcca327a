// k_search.cu -- exact lattice k-NN on the device: quantization, a tensor-core distance bound over
// the high parts of the components, exact re-scoring of the candidates, exact scans where the bound
// cannot decide.
//
// Semantics (the reference's embed+search path):
//   * components: EmbeddingAdapter.QuantizeDense (Math/EmbeddingAdapter.cs:43-54), equal entry for
//     entry to the dense form of Quantize (:15-41) without a sparsity budget: |e| < ZeroThreshold
//     (float compare) -> 0, else (long)(e * (double)GlobalScale). Stored as int32; a component
//     outside int32 is an error (ERANGE).
//   * distance: SparseVector.DistanceSquaredL2Fast (Math/SparseVector.cs:138-169) on the dense rows,
//     sum of (ulong)(diff * diff) with wrap-around.
//   * result: the k smallest (distance, row) pairs, ascending. The reference orders equal distances
//     by an unstable sort (RecallEvaluator.cs:148-163, KnnHeap EmbeddingLattice.cs:321-387); here
//     they are ordered by row id.
//
// Bound. Every component is split v = v_h * 2^s + v_l with |v_l| <= 2^(s-1) and v_h a two-digit
// balanced base-256 integer (s per side from its largest |v|). One kind::i8 tcgen05 pass computes
// H = q_h . d_h exactly (2 x 2 digit products per pair, int32 in TMEM), so
//     approx(q, d) = |q|^2 + |d|^2 - 2^(sq+sd+1) H,   |dist - approx| <= E(q)
//     E(q) = 2 (2^sq |q_h| L + 2^sd |q_l| H_max + |q_l| L),  L = max |d_l|, H_max = max |d_h|
// (Cauchy-Schwarz; norms rounded up). Each (query, slot) keeps the T smallest approx keys; the merge
// re-scores the T best candidates exactly and accepts the answer when the T-th smallest approx
// distance minus E(q) exceeds the k-th exact distance, which rules out every other row. Otherwise
// (or when |q| + |d| might reach 2^31, where the key arithmetic could overflow) the query is
// answered by an exact scan of every row.
#include <cuda.h>

#include <algorithm>
#include <cmath>
#include <cstring>

#include "slx_attr.h"
#include "slx_device.cuh"
#include "slx_gemm.h"
#include "slx_kernels.h"
#include "slx_search.h"
#include "slx_status.h"
#include "tc_ptx.cuh"

namespace slx {
namespace search {
namespace {

using namespace tc;

constexpr int QBM = 128;   // queries per tile (TMEM lanes)
constexpr int DBN = 80;    // database rows per tile: 3 column blocks of 80 per accumulator, two accumulators
constexpr int BKB = 128;   // K bytes per ring stage (one 128-byte swizzle row)
constexpr int STAGES = 3;
constexpr int THREADS = 320;  // warp 0 TMA, warp 1 TMEM + MMA, warps 2..9 epilogue
constexpr int EPI = 256;      // epilogue threads
constexpr int A_STAGE = 2 * QBM * BKB;
constexpr int B_STAGE = 2 * DBN * BKB;
constexpr int STAGE = A_STAGE + B_STAGE;
constexpr int ACC_COLS = 256;  // TMEM column stride of the two accumulators
constexpr int HALF = DBN / 2;  // database columns per epilogue warp
constexpr int CAP = 16;        // pending candidates per epilogue thread
constexpr size_t BUF_BYTES = (size_t)CAP * EPI * 12;
constexpr size_t SMEM = (size_t)STAGES * STAGE + BUF_BYTES + 1024 + 256;
static_assert(STAGE % 1024 == 0 && A_STAGE % 1024 == 0, "swizzle atoms stay 1024-byte aligned");
static_assert(3 * DBN <= ACC_COLS && ACC_COLS + 3 * DBN <= 512, "two accumulators in 512 TMEM columns");
static_assert(HALF % 8 == 0, "epilogue chunks of 8 columns");
constexpr int EXACT_THREADS = 256;

SLX_DEV int pick_shift(unsigned long long max_abs) {
    int s = 0;
    while (s < 40) {
        const unsigned long long h = s ? (max_abs + (1ull << (s - 1))) >> s : max_abs;
        if (h <= 32639ull) break;  // two balanced base-256 digits
        s++;
    }
    return s;
}

// |q| + |d| < 2^31 for every pair: every distance, norm and key then stays below 2^62.
SLX_DEV bool bound_ok(const SideStats* qs, const SideStats* ds) {
    return sqrt((double)qs->max_norm2) + sqrt((double)ds->max_norm2) < 2147483647.0;
}

SLX_DEV bool less_pair(int64_t ka, int32_t ia, int64_t kb, int32_t ib) { return ka < kb || (ka == kb && ia < ib); }

// Keeps the T smallest (key, id) pairs: replace the current largest, then find the new largest.
SLX_DEV void list_put(int64_t (&lk)[T], int32_t (&li)[T], int64_t& wk, int32_t& wi, int& wp, int64_t key, int32_t id) {
#pragma unroll
    for (int j = 0; j < T; j++)
        if (j == wp) { lk[j] = key; li[j] = id; }
    wk = lk[0]; wi = li[0]; wp = 0;
#pragma unroll
    for (int j = 1; j < T; j++)
        if (less_pair(wk, wi, lk[j], li[j])) { wk = lk[j]; wi = li[j]; wp = j; }
}

// ---- quantization and digit split ----

__global__ void k_quantize(const float* __restrict__ x, int64_t total, float thr, double scale, int32_t* __restrict__ out,
                           SideStats* stats) {
    unsigned long long mx = 0;
    int bad = 0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const float e = x[i];
        int64_t v = fabsf(e) < thr ? 0 : cs_d2l(__dmul_rn((double)e, scale));
        if (v < INT32_MIN || v > INT32_MAX) { bad = 1; v = 0; }
        out[i] = (int32_t)v;
        const unsigned long long a = (unsigned long long)(v < 0 ? -v : v);
        mx = a > mx ? a : mx;
    }
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long w = __shfl_xor_sync(0xffffffffu, mx, o);
        mx = w > mx ? w : mx;
    }
    bad = __any_sync(0xffffffffu, bad);
    if ((threadIdx.x & 31) == 0) {
        if (mx) atomicMax(&stats->max_abs, mx);
        if (bad) atomicExch(&stats->range_bad, 1);
    }
}

// One warp per row: digit planes of the high parts, exact squared norms of the row and of its parts.
__global__ void k_split(const int32_t* __restrict__ vals, int64_t n, int dim, int64_t npad, int dpad,
                        int8_t* __restrict__ planes, uint64_t* __restrict__ norm2, uint64_t* __restrict__ h2,
                        uint64_t* __restrict__ l2, SideStats* stats) {
    const int s = pick_shift(stats->max_abs);
    const int lane = threadIdx.x & 31;
    const int64_t row = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= n) return;
    u128 nn = 0;
    uint64_t hh = 0, ll = 0;
    const int32_t* src = vals + row * dim;
    int8_t* p0 = planes + row * dpad;
    int8_t* p1 = p0 + npad * dpad;
    for (int d = lane; d < dim; d += 32) {
        const int64_t v = src[d];
        const int64_t h = s ? (v + (1LL << (s - 1))) >> s : v;
        const int64_t l = v - h * (1LL << s);
        const int d0 = (int)(((uint64_t)h + 128u) & 255u) - 128;
        const int d1 = (int)((h - d0) >> 8);
        p0[d] = (int8_t)d0;
        p1[d] = (int8_t)d1;
        nn += (u128)(uint64_t)(v * v);
        hh += (uint64_t)(h * h);
        ll += (uint64_t)(l * l);
    }
    nn = warp_sum_u128(nn);
    for (int o = 16; o > 0; o >>= 1) {
        hh += __shfl_xor_sync(0xffffffffu, (unsigned long long)hh, o);
        ll += __shfl_xor_sync(0xffffffffu, (unsigned long long)ll, o);
    }
    if (lane == 0) {
        const uint64_t ns = nn >= ((u128)1 << 63) ? (1ull << 63) : (uint64_t)nn;
        norm2[row] = ns;
        if (h2) { h2[row] = hh; l2[row] = ll; }
        atomicMax(&stats->max_norm2, (unsigned long long)ns);
        atomicMax(&stats->max_h2, (unsigned long long)hh);
        atomicMax(&stats->max_l2, (unsigned long long)ll);
    }
}

// ---- tensor-core bound pass ----

struct TcParams {
    int nq, nkb, tiles_per_chunk, ntiles, nslots;
    int64_t n;
    const uint64_t* dn;
    const SideStats* qs;
    const SideStats* ds;
    int64_t* ckey;  // [nq][nslots][T]
    int32_t* cid;
    int* err;
};

// CTA = 128 queries x one chunk of database tiles (80 rows each). Per tile, for every 32-byte K step,
// two MMAs (M=128, N=160, K=32): query digit i times the database's two digit planes stacked along N,
// written at TMEM column 80*i of the tile's accumulator, so products of digit sum i+j accumulate in
// column block i+j. Tiles alternate between two accumulators (columns 0 and 256), so the epilogue
// of one tile overlaps the MMAs of the next. The first MMA of a tile overwrites blocks 0 and 1;
// block 2 is cleared by the epilogue after it reads the tile.
// Epilogue warps: lane quadrant warp%4, column half (warp-2)/4. Each thread keeps its query's T
// smallest keys over the chunk; keys under the thread's threshold queue in shared memory and the
// warp merges the queues together, so one pass over the list code serves many lanes.
__global__ void __launch_bounds__(THREADS, 1)
k_search_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmD, TcParams p) {
    constexpr uint32_t IDESC = idesc_i8(2 * DBN);
    if (!bound_ok(p.qs, p.ds)) return;  // the merge sends every query to the exact scan
    if ((int)blockIdx.y * p.tiles_per_chunk >= p.ntiles) return;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    int64_t* q_key = (int64_t*)(smem + (size_t)STAGES * STAGE);  // [CAP][EPI]
    int32_t* q_id = (int32_t*)(q_key + CAP * EPI);                // [CAP][EPI]
    uint64_t* bars = (uint64_t*)(smem + (size_t)STAGES * STAGE + BUF_BYTES);
    const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * STAGES;
    const uint32_t tfull0 = empty0 + 8 * STAGES, tempty0 = tfull0 + 16;  // two each
    uint32_t* tmem_slot = (uint32_t*)(bars + 2 * STAGES + 4);
    __shared__ int s_fail;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        s_fail = 0;
        for (int i = 0; i < STAGES; i++) {
            mbar_init(full0 + 8 * i, 1);
            mbar_init(empty0 + 8 * i, 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(tfull0 + 8 * b, 1);
            mbar_init(tempty0 + 8 * b, 8);
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
    if (warp >= 2 && warp < 6) {  // column block 2 of both accumulators starts at zero
        const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
#pragma unroll
        for (int b = 0; b < 2; b++) {
#pragma unroll
            for (int c = 0; c < DBN; c += 16) tmem_st16_zero(tmem + lane_base + b * ACC_COLS + 2 * DBN + c);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    fence_before();
    __syncthreads();
    fence_after();

    // blockIdx.x = query tile (fastest), blockIdx.y = database chunk: the CTAs resident together are
    // the query tiles of one or two chunks, which then read the same database tiles through L2.
    const int m0 = blockIdx.x * QBM;
    const int t0 = blockIdx.y * p.tiles_per_chunk;
    const int ntl = min(p.tiles_per_chunk, p.ntiles - t0);
    const uint32_t sbase = smem_u32(smem);

    if (warp == 0) {
        if (lane == 0) {  // TMA producer
            const int total = ntl * p.nkb;
            int issued = 0;
            for (int it = 0; it < total; it++) {
                const int s = it % STAGES;
                const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
                if (!mbar_wait(empty0 + 8 * s, ph ^ 1u)) { s_fail = 1; break; }
                if (*(volatile int*)&s_fail) break;
                const int t = t0 + it / p.nkb, kb = it % p.nkb;
                mbar_expect_tx(full0 + 8 * s, STAGE);
                tma_load_4d(sbase + s * STAGE, &tmQ, kb * BKB, m0, 0, 0, full0 + 8 * s);
                tma_load_4d(sbase + s * STAGE + A_STAGE, &tmD, kb * BKB, t * DBN, 0, 0, full0 + 8 * s);
                issued = it + 1;
            }
            if (*(volatile int*)&s_fail) {  // let copies still in flight land before the CTA exits
                for (int it = issued - STAGES < 0 ? 0 : issued - STAGES; it < issued; it++)
                    mbar_wait(full0 + 8 * (it % STAGES), (uint32_t)(it / STAGES) & 1u);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            int it = 0;
            for (int j = 0; j < ntl; j++) {
                const int b = j & 1;
                if (!mbar_wait(tempty0 + 8 * b, (uint32_t)((j >> 1) & 1) ^ 1u)) { s_fail = 1; break; }
                fence_after();
                const uint32_t acc = tmem + b * ACC_COLS;
                bool fail = false;
                for (int kb = 0; kb < p.nkb; kb++, it++) {
                    const int s = it % STAGES;
                    if (!mbar_wait(full0 + 8 * s, (uint32_t)(it / STAGES) & 1u)) { fail = true; break; }
                    fence_after();
                    const uint32_t a = sbase + s * STAGE, bb = a + A_STAGE;
#pragma unroll
                    for (int kk = 0; kk < BKB / 32; kk++) {
                        const uint64_t bdesc = sw128_desc(bb + kk * 32);
#pragma unroll
                        for (int i = 0; i < 2; i++)
                            umma_i8(acc + i * DBN, sw128_desc(a + i * (QBM * BKB) + kk * 32), bdesc, IDESC,
                                    (kb | kk | i) ? 1u : 0u);
                    }
                    umma_commit(empty0 + 8 * s);
                }
                if (fail) { s_fail = 1; break; }
                umma_commit(tfull0 + 8 * b);
            }
        }
    } else {  // epilogue
        const int quad = warp & 3, half = (warp - 2) >> 2;
        const int et = threadIdx.x - 64;  // epilogue thread index
        const int row = m0 + 32 * quad + lane;
        const uint32_t taddr = tmem + ((uint32_t)(32 * quad) << 16);
        const int sh = pick_shift(p.qs->max_abs) + pick_shift(p.ds->max_abs) + 1;
        int64_t lk[T];
        int32_t li[T];
#pragma unroll
        for (int j = 0; j < T; j++) { lk[j] = INT64_MAX; li[j] = INT32_MAX; }
        int64_t wk = INT64_MAX;
        int32_t wi = INT32_MAX;
        int wp = 0, cnt = 0;
        auto flush = [&]() {
            const int mx = __reduce_max_sync(0xffffffffu, cnt);
            for (int i = 0; i < mx; i++) {
                if (i < cnt) {
                    const int64_t key = q_key[i * EPI + et];
                    const int32_t id = q_id[i * EPI + et];
                    if (less_pair(key, id, wk, wi)) list_put(lk, li, wk, wi, wp, key, id);
                }
            }
            cnt = 0;
        };
        bool ok = true;
        for (int j = 0; j < ntl; j++) {
            const int b = j & 1;
            const int64_t nbase = (int64_t)(t0 + j) * DBN + HALF * half;
            // this tile's squared norms, fetched before the wait: lane l holds columns l and 32 + l
            const int64_t dn0 = (int64_t)__ldg(p.dn + min(nbase + lane, p.n - 1));
            const int64_t dn1 = lane + 32 < HALF ? (int64_t)__ldg(p.dn + min(nbase + 32 + lane, p.n - 1)) : 0;
            ok = __all_sync(0xffffffffu, mbar_wait(tfull0 + 8 * b, (uint32_t)(j >> 1) & 1u));  // tcgen05.ld is warp-collective
            if (!ok) { s_fail = 1; break; }
            fence_after();
            const uint32_t acc = taddr + b * ACC_COLS + HALF * half;
#pragma unroll 1
            for (int c = 0; c < HALF / 8; c++) {
                uint32_t g0[8], g1[8], g2[8];
                tmem_ld8(acc + 8 * c, g0);
                tmem_ld8(acc + DBN + 8 * c, g1);
                tmem_ld8(acc + 2 * DBN + 8 * c, g2);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int jj = 0; jj < 8; jj++) {
                    const int col = 8 * c + jj;
                    const int64_t dnc = (int64_t)__shfl_sync(0xffffffffu, (long long)(col < 32 ? dn0 : dn1), col & 31);
                    const int64_t n = nbase + col;
                    const int64_t h = (int64_t)(int32_t)g0[jj] + (int64_t)(int32_t)g1[jj] * 256 +
                                      (int64_t)(int32_t)g2[jj] * 65536;
                    const int64_t key = wsub(dnc, (int64_t)((uint64_t)h << sh));
                    if (n < p.n && less_pair(key, (int32_t)n, wk, wi)) {
                        q_key[cnt * EPI + et] = key;
                        q_id[cnt * EPI + et] = (int32_t)n;
                        cnt++;
                    }
                }
                if (__any_sync(0xffffffffu, cnt > CAP - 8)) flush();
            }
#pragma unroll
            for (int c = 0; c < HALF; c += 8) tmem_st8_zero(taddr + b * ACC_COLS + 2 * DBN + HALF * half + c);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty0 + 8 * b);
        }
        flush();
        if (ok && row < p.nq) {
            const size_t base = ((size_t)row * p.nslots + (size_t)blockIdx.y * 2 + half) * T;
#pragma unroll
            for (int j = 0; j < T; j++) { p.ckey[base + j] = lk[j]; p.cid[base + j] = li[j]; }
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

// ---- exact scan ----

// Block = one query x one chunk of rows; each warp keeps the T smallest (distance, row) of its rows.
// Keys are distance ^ 2^63 so that int64 order is distance order.
__global__ void __launch_bounds__(EXACT_THREADS)
k_search_exact(const int32_t* __restrict__ dvals, int64_t n, int dim, const int32_t* __restrict__ qvals,
               const int* __restrict__ qlist, int64_t rows_per_chunk, int nslots, int64_t* __restrict__ ckey,
               int32_t* __restrict__ cid) {
    extern __shared__ int32_t s_q[];
    const int f = blockIdx.y;
    const int q = qlist ? qlist[f] : f;
    for (int d = threadIdx.x; d < dim; d += blockDim.x) s_q[d] = qvals[(int64_t)q * dim + d];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int64_t r0 = blockIdx.x * rows_per_chunk, r1 = min(r0 + rows_per_chunk, n);
    int64_t lk[T];
    int32_t li[T];
#pragma unroll
    for (int j = 0; j < T; j++) { lk[j] = INT64_MAX; li[j] = INT32_MAX; }
    int64_t wk = INT64_MAX;
    int32_t wi = INT32_MAX;
    int wp = 0;
    for (int64_t r = r0 + warp; r < r1; r += nw) {
        const int32_t* row = dvals + r * dim;
        uint64_t s = 0;
        for (int d = lane; d < dim; d += 32) {
            const int64_t diff = (int64_t)s_q[d] - (int64_t)row[d];
            const uint64_t ad = (uint64_t)(diff < 0 ? -diff : diff);
            s += ad * ad;  // (ulong)(diff * diff)
        }
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, (unsigned long long)s, o);
        const int64_t key = (int64_t)(s ^ (1ull << 63));
        if (lane == 0 && less_pair(key, (int32_t)r, wk, wi)) list_put(lk, li, wk, wi, wp, key, (int32_t)r);
    }
    if (lane == 0) {
        const size_t base = ((size_t)f * nslots + (size_t)blockIdx.x * nw + warp) * T;
#pragma unroll
        for (int j = 0; j < T; j++) { ckey[base + j] = lk[j]; cid[base + j] = li[j]; }
    }
}

// ---- merge ----

struct MergeParams {
    int nslots, k, mode;  // mode 0: bound candidates (re-score, certify); 1: exact lists
    const int64_t* ckey;
    const int32_t* cid;
    const int* qlist;  // mode 1: query of list row (null: identity)
    const int32_t* qvals;
    const int32_t* dvals;
    int dim;
    const uint64_t* qn2;
    const uint64_t* qh2;
    const uint64_t* ql2;
    const SideStats* qs;
    const SideStats* ds;
    int64_t n, id_base;
    const int32_t* payload;  // ids are payload[row] when set, else id_base + row
    int64_t* out_ids;
    uint64_t* out_dist;
    int* fb_list;
    int* fb_count;
};

constexpr int MT = 128;  // merge threads

__global__ void __launch_bounds__(MT) k_search_merge(MergeParams p) {
    __shared__ int64_t s_key[MT][T];
    __shared__ int32_t s_id[MT][T];
    __shared__ int64_t r_key[MT / 32];
    __shared__ int32_t r_id[MT / 32];
    __shared__ int r_thr[MT / 32];
    __shared__ int64_t sel_key[T];
    __shared__ int32_t sel_id[T];
    __shared__ uint64_t sel_dist[T];
    const int r = blockIdx.x;
    const int q = (p.mode == 1 && p.qlist) ? p.qlist[r] : r;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (p.mode == 0 && !bound_ok(p.qs, p.ds)) {  // the bound pass did not run
        if (tid == 0) p.fb_list[atomicAdd(p.fb_count, 1)] = q;
        return;
    }
    // this thread's T smallest entries of the row
    {
        int64_t lk[T];
        int32_t li[T];
#pragma unroll
        for (int j = 0; j < T; j++) { lk[j] = INT64_MAX; li[j] = INT32_MAX; }
        int64_t wk = INT64_MAX;
        int32_t wi = INT32_MAX;
        int wp = 0;
        const int64_t tot = (int64_t)p.nslots * T;
        const int64_t* kr = p.ckey + (size_t)r * tot;
        const int32_t* ir = p.cid + (size_t)r * tot;
        for (int64_t e = tid; e < tot; e += MT) {
            const int64_t key = kr[e];
            const int32_t id = ir[e];
            if (less_pair(key, id, wk, wi)) list_put(lk, li, wk, wi, wp, key, id);
        }
#pragma unroll
        for (int j = 0; j < T; j++) { s_key[tid][j] = lk[j]; s_id[tid][j] = li[j]; }
    }
    __syncthreads();
    // T rounds of block-wide minimum
    for (int round = 0; round < T; round++) {
        int64_t bk = INT64_MAX;
        int32_t bi = INT32_MAX;
        int bj = 0;
        for (int j = 0; j < T; j++)
            if (less_pair(s_key[tid][j], s_id[tid][j], bk, bi)) { bk = s_key[tid][j]; bi = s_id[tid][j]; bj = j; }
        int bt = tid;
        for (int o = 16; o > 0; o >>= 1) {
            const int64_t ok = (int64_t)__shfl_xor_sync(0xffffffffu, (long long)bk, o);
            const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            const int ot = __shfl_xor_sync(0xffffffffu, bt, o);
            if (less_pair(ok, oi, bk, bi) || (ok == bk && oi == bi && ot < bt)) { bk = ok; bi = oi; bt = ot; }
        }
        if (lane == 0) { r_key[warp] = bk; r_id[warp] = bi; r_thr[warp] = bt; }
        __syncthreads();
        if (tid == 0) {
            int64_t k0 = r_key[0];
            int32_t i0 = r_id[0];
            int t0 = r_thr[0];
            for (int w = 1; w < MT / 32; w++)
                if (less_pair(r_key[w], r_id[w], k0, i0)) { k0 = r_key[w]; i0 = r_id[w]; t0 = r_thr[w]; }
            sel_key[round] = k0;
            sel_id[round] = i0;
            r_thr[0] = t0;
        }
        __syncthreads();
        if (tid == r_thr[0] && bk == sel_key[round] && bi == sel_id[round]) {
            s_key[tid][bj] = INT64_MAX;
            s_id[tid][bj] = INT32_MAX;
        }
        __syncthreads();
    }

    if (p.mode == 1) {  // exact lists: keys are distance ^ 2^63
        if (tid < p.k) {
            const bool valid = sel_id[tid] != INT32_MAX;
            p.out_ids[(size_t)q * p.k + tid] =
                valid ? (p.payload ? (int64_t)p.payload[sel_id[tid]] : p.id_base + sel_id[tid]) : -1;
            p.out_dist[(size_t)q * p.k + tid] = valid ? ((uint64_t)sel_key[tid] ^ (1ull << 63)) : UINT64_MAX;
        }
        return;
    }

    // exact distances of the T candidates: warp w scores candidates w, w+4, ...
    for (int c = warp; c < T; c += MT / 32) {
        const int32_t id = sel_id[c];
        uint64_t s = UINT64_MAX;
        if (id != INT32_MAX) {
            const int32_t* a = p.qvals + (size_t)q * p.dim;
            const int32_t* b = p.dvals + (size_t)id * p.dim;
            s = 0;
            for (int d = lane; d < p.dim; d += 32) {
                const int64_t diff = (int64_t)a[d] - (int64_t)b[d];
                const uint64_t ad = (uint64_t)(diff < 0 ? -diff : diff);
                s += ad * ad;
            }
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, (unsigned long long)s, o);
        }
        if (lane == 0) sel_dist[c] = s;
    }
    __syncthreads();
    if (tid == 0) {
        uint64_t dd[T];
        int32_t di[T];
        int nv = 0;
        for (int c = 0; c < T; c++) {  // insertion sort by (distance, id)
            if (sel_id[c] == INT32_MAX) continue;
            uint64_t dv = sel_dist[c];
            int32_t iv = sel_id[c];
            int j = nv++;
            while (j > 0 && (dd[j - 1] > dv || (dd[j - 1] == dv && di[j - 1] > iv))) {
                dd[j] = dd[j - 1];
                di[j] = di[j - 1];
                j--;
            }
            dd[j] = dv;
            di[j] = iv;
        }
        bool certified = nv < T;  // fewer than T rows in the database: every row was scored
        if (!certified) {
            const int sq = pick_shift(p.qs->max_abs), sd = pick_shift(p.ds->max_abs);
            const double qh = __dsqrt_ru((double)p.qh2[q]), ql = __dsqrt_ru((double)p.ql2[q]);
            const double hb = __dsqrt_ru((double)p.ds->max_h2), lb = __dsqrt_ru((double)p.ds->max_l2);
            const double e = __dadd_ru(__dadd_ru(__dmul_ru(__dmul_ru(ldexp(1.0, sq), qh), lb),
                                                 __dmul_ru(__dmul_ru(ldexp(1.0, sd), ql), hb)),
                                       __dmul_ru(ql, lb));
            const double E = ceil(__dmul_ru(2.0, e)) + 1.0;
            if (E < 4.0e18) {
                const i128 lower = (i128)p.qn2[q] + (i128)sel_key[T - 1] - (i128)(int64_t)E;
                certified = lower > (i128)dd[p.k - 1];
            }
        }
        if (certified) {
            for (int j = 0; j < p.k; j++) {
                const bool valid = j < nv;
                p.out_ids[(size_t)q * p.k + j] = valid ? (p.payload ? (int64_t)p.payload[di[j]] : p.id_base + di[j]) : -1;
                p.out_dist[(size_t)q * p.k + j] = valid ? dd[j] : UINT64_MAX;
            }
        } else {
            p.fb_list[atomicAdd(p.fb_count, 1)] = q;
        }
    }
}

// Ascending merge of `parts` sorted top-k lists per query; id -1 marks an empty entry.
__global__ void k_merge_parts(const int64_t* __restrict__ ids, const uint64_t* __restrict__ dist, int parts, int nq, int k,
                              int64_t* __restrict__ oi, uint64_t* __restrict__ od) {
    const int q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= nq) return;
    int ptr[64];
    for (int pp = 0; pp < parts; pp++) ptr[pp] = 0;
    for (int j = 0; j < k; j++) {
        int best = -1;
        uint64_t bd = UINT64_MAX;
        uint64_t bid = UINT64_MAX;
        for (int pp = 0; pp < parts; pp++) {
            if (ptr[pp] >= k) continue;
            const size_t e = ((size_t)pp * nq + q) * k + ptr[pp];
            if (ids[e] < 0) continue;
            const uint64_t d = dist[e], id = (uint64_t)ids[e];
            if (best < 0 || d < bd || (d == bd && id < bid)) { best = pp; bd = d; bid = id; }
        }
        if (best < 0) {
            oi[(size_t)q * k + j] = -1;
            od[(size_t)q * k + j] = UINT64_MAX;
        } else {
            oi[(size_t)q * k + j] = (int64_t)bid;
            od[(size_t)q * k + j] = bd;
            ptr[best]++;
        }
    }
}

int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

template <class P>
P* carve(uint8_t*& cur, size_t count) {
    P* p = (P*)cur;
    cur += (count * sizeof(P) + 255) & ~(size_t)255;
    return p;
}

unsigned grid_for(int64_t total, int threads) {
    int64_t b = (total + threads - 1) / threads;
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>(b, 148 * 16));
}

// Chunks per query tile minimizing (waves of 148 CTAs) x (tiles per CTA), with chunks of at least
// MIN_CHUNK tiles when the database has them: a slot's first candidates all enter its list, so short
// chunks pay that start-up on every CTA.
constexpr int MIN_CHUNK = 256;
int pick_chunks(int qtiles, int ntiles) {
    int best = 1;
    double best_cost = 1e300;
    const int maxc = std::max(1, std::min(ntiles / MIN_CHUNK, 4096));
    for (int c = 1; c <= maxc; c++) {
        const int per = (ntiles + c - 1) / c;
        const int chunks = (ntiles + per - 1) / per;
        const double waves = std::ceil((double)qtiles * chunks / 148.0);
        const double cost = waves * per;
        if (cost < best_cost - 1e-9) { best_cost = cost; best = chunks; }
    }
    return best;
}

}  // namespace

int build(const float* d_vectors, int64_t n, int dim, float zero_threshold, int64_t global_scale, int64_t id_base,
          Lattice& L, cudaStream_t st, std::string& err) {
    if (n < 0 || dim < 1 || dim > MAX_DIM || n > INT32_MAX - 256) { err = "lattice: bad shape"; return SLX_EINVAL; }
    if (n > 0 && !d_vectors) { err = "lattice: null vectors"; return SLX_EINVAL; }
    cudaGetDevice(&L.device);
    L.n = n;
    L.dim = dim;
    L.dpad = (int)round_up(dim, BKB);
    L.npad = round_up(std::max<int64_t>(n, 1), DBN);
    L.id_base = id_base;
    const size_t vbytes = (size_t)n * dim * 4, pbytes = (size_t)2 * L.npad * L.dpad;
    if (cudaMalloc(&L.stats, sizeof(SideStats)) != cudaSuccess || cudaMalloc(&L.counters, 256) != cudaSuccess ||
        cudaMalloc(&L.planes, pbytes) != cudaSuccess || cudaMalloc(&L.norm2, (size_t)L.npad * 8) != cudaSuccess ||
        (vbytes && cudaMalloc(&L.vals, vbytes) != cudaSuccess)) {
        cudaGetLastError();
        err = "lattice: device allocation failed";
        return SLX_EOOM;
    }
    cudaMemsetAsync(L.stats, 0, sizeof(SideStats), st);
    cudaMemsetAsync(L.planes, 0, pbytes, st);
    if (n > 0) {
        k_quantize<<<grid_for(n * dim, 256), 256, 0, st>>>(d_vectors, n * dim, zero_threshold, (double)global_scale,
                                                           L.vals, L.stats);
        k_split<<<(unsigned)((n + 7) / 8), 256, 0, st>>>(L.vals, n, dim, L.npad, L.dpad, L.planes, L.norm2, nullptr,
                                                         nullptr, L.stats);
    }
    SideStats hs;
    cudaMemcpyAsync(&hs, L.stats, sizeof(hs), cudaMemcpyDeviceToHost, st);
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) { err = cudaGetErrorString(e); return SLX_ECUDA; }
    if (hs.range_bad) { err = "lattice: a quantized component does not fit 32 bits"; return SLX_ERANGE; }
    if (!tc::encode_planes(L.tmap, L.planes, L.dpad, L.npad, 2, DBN)) { err = "lattice: tensor map"; return SLX_ECUDA; }
    return SLX_OK;
}

// Max |component| of int32 rows (the quantize kernel's statistic, for rows quantized elsewhere).
__global__ void k_maxabs(const int32_t* __restrict__ v, int64_t total, SideStats* stats) {
    unsigned long long mx = 0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t x = v[i];
        const unsigned long long a = (unsigned long long)(x < 0 ? -x : x);
        mx = a > mx ? a : mx;
    }
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long w = __shfl_xor_sync(0xffffffffu, mx, o);
        mx = w > mx ? w : mx;
    }
    if ((threadIdx.x & 31) == 0 && mx) atomicMax(&stats->max_abs, mx);
}

int build_quantized(const int32_t* d_rows, int64_t n, int dim, int64_t id_base, Lattice& L, cudaStream_t st,
                    std::string& err) {
    if (n < 0 || dim < 1 || dim > MAX_DIM || n > INT32_MAX - 256) { err = "lattice: bad shape"; return SLX_EINVAL; }
    cudaGetDevice(&L.device);
    L.n = n;
    L.dim = dim;
    L.dpad = (int)round_up(dim, BKB);
    L.npad = round_up(std::max<int64_t>(n, 1), DBN);
    L.id_base = id_base;
    const size_t vbytes = (size_t)n * dim * 4, pbytes = (size_t)2 * L.npad * L.dpad;
    if (cudaMalloc(&L.stats, sizeof(SideStats)) != cudaSuccess || cudaMalloc(&L.counters, 256) != cudaSuccess ||
        cudaMalloc(&L.planes, pbytes) != cudaSuccess || cudaMalloc(&L.norm2, (size_t)L.npad * 8) != cudaSuccess ||
        (vbytes && cudaMalloc(&L.vals, vbytes) != cudaSuccess)) {
        cudaGetLastError();
        err = "lattice: device allocation failed";
        return SLX_EOOM;
    }
    cudaMemsetAsync(L.stats, 0, sizeof(SideStats), st);
    cudaMemsetAsync(L.planes, 0, pbytes, st);
    if (n > 0) {
        cudaMemcpyAsync(L.vals, d_rows, vbytes, cudaMemcpyDeviceToDevice, st);
        k_maxabs<<<grid_for(n * dim, 256), 256, 0, st>>>(L.vals, n * dim, L.stats);
        k_split<<<(unsigned)((n + 7) / 8), 256, 0, st>>>(L.vals, n, dim, L.npad, L.dpad, L.planes, L.norm2, nullptr,
                                                         nullptr, L.stats);
    }
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) { err = cudaGetErrorString(e); return SLX_ECUDA; }
    if (!tc::encode_planes(L.tmap, L.planes, L.dpad, L.npad, 2, DBN)) { err = "lattice: tensor map"; return SLX_ECUDA; }
    return SLX_OK;
}

void release(Lattice& L) {
    cudaFree(L.payload);
    cudaFree(L.vals);
    cudaFree(L.planes);
    cudaFree(L.norm2);
    cudaFree(L.stats);
    cudaFree(L.counters);
    cudaFree(L.qws);
    cudaFree(L.xws);
    L = Lattice();
}

int query(Lattice& L, const float* d_q, int nq, int k, float zero_threshold, int64_t global_scale, bool exact_only,
          int64_t* d_ids, uint64_t* d_dist, int* n_fallback, cudaStream_t st, std::string& err, int64_t* launches) {
    if (n_fallback) *n_fallback = 0;
    if (nq < 0 || k < 0 || k > KMAX) { err = "lattice query: k must be in [0, 16]"; return SLX_EINVAL; }
    if (nq == 0 || k == 0) return SLX_OK;
    if (!d_q || !d_ids || !d_dist) { err = "lattice query: null buffer"; return SLX_EINVAL; }
    if (L.n == 0) {
        cudaMemsetAsync(d_ids, 0xFF, (size_t)nq * k * 8, st);
        cudaMemsetAsync(d_dist, 0xFF, (size_t)nq * k * 8, st);
        return SLX_OK;
    }
    const int dim = L.dim, dpad = L.dpad;
    const int64_t qpad = round_up(nq, QBM);
    const int qtiles = (int)(qpad / QBM), ntiles = (int)(L.npad / DBN);
    const int nchunks = exact_only ? 1 : pick_chunks(qtiles, ntiles);
    const int per = (ntiles + nchunks - 1) / nchunks;
    const int nslots = 2 * nchunks;
    // scratch
    const size_t need = ((size_t)nq * dim * 4 + 256) + ((size_t)2 * qpad * dpad + 256) + 3 * ((size_t)qpad * 8 + 256) +
                        (sizeof(SideStats) + 256) + ((size_t)nq * nslots * T * 12 + 512) + ((size_t)nq * 4 + 256) + 1024;
    if (need > L.qws_bytes) {
        cudaFree(L.qws);
        L.qws = nullptr;
        L.qws_bytes = 0;
        if (cudaMalloc(&L.qws, need) != cudaSuccess) { cudaGetLastError(); err = "lattice query: scratch"; return SLX_EOOM; }
        L.qws_bytes = need;
    }
    uint8_t* cur = (uint8_t*)L.qws;
    int32_t* qvals = carve<int32_t>(cur, (size_t)nq * dim);
    int8_t* qplanes = carve<int8_t>(cur, (size_t)2 * qpad * dpad);
    uint64_t* qn2 = carve<uint64_t>(cur, qpad);
    uint64_t* qh2 = carve<uint64_t>(cur, qpad);
    uint64_t* ql2 = carve<uint64_t>(cur, qpad);
    SideStats* qs = carve<SideStats>(cur, 1);
    int64_t* ckey = carve<int64_t>(cur, (size_t)nq * nslots * T);
    int32_t* cid = carve<int32_t>(cur, (size_t)nq * nslots * T);
    int* fb_list = carve<int>(cur, nq);

    int64_t nl = 0;
    cudaMemsetAsync(qs, 0, sizeof(SideStats), st);
    cudaMemsetAsync(L.counters, 0, 256, st);
    k_quantize<<<grid_for((int64_t)nq * dim, 256), 256, 0, st>>>(d_q, (int64_t)nq * dim, zero_threshold,
                                                                 (double)global_scale, qvals, qs);
    nl++;
    if (!exact_only) {
        cudaMemsetAsync(qplanes, 0, (size_t)2 * qpad * dpad, st);
        k_split<<<(unsigned)((nq + 7) / 8), 256, 0, st>>>(qvals, nq, dim, qpad, dpad, qplanes, qn2, qh2, ql2, qs);
        alignas(64) unsigned char tmq[128];
        if (!tc::encode_planes(tmq, qplanes, dpad, qpad, 2, QBM)) { err = "lattice query: tensor map"; return SLX_ECUDA; }
        slx::ensure_smem((const void*)k_search_tc, SMEM);
        TcParams tp;
        tp.nq = nq; tp.nkb = dpad / BKB; tp.tiles_per_chunk = per; tp.ntiles = ntiles; tp.nslots = nslots;
        tp.n = L.n; tp.dn = L.norm2; tp.qs = qs; tp.ds = L.stats; tp.ckey = ckey; tp.cid = cid;
        tp.err = L.counters + 2;
        CUtensorMap mq, md;
        memcpy(&mq, tmq, sizeof(mq));
        memcpy(&md, L.tmap, sizeof(md));
        k_search_tc<<<dim3((unsigned)qtiles, (unsigned)nchunks), THREADS, SMEM, st>>>(mq, md, tp);
        MergeParams mp{};
        mp.nslots = nslots; mp.k = k; mp.mode = 0; mp.ckey = ckey; mp.cid = cid; mp.qlist = nullptr;
        mp.qvals = qvals; mp.dvals = L.vals; mp.dim = dim; mp.qn2 = qn2; mp.qh2 = qh2; mp.ql2 = ql2;
        mp.qs = qs; mp.ds = L.stats; mp.n = L.n; mp.id_base = L.id_base; mp.out_ids = d_ids; mp.out_dist = d_dist;
        mp.payload = L.payload;
        mp.fb_list = fb_list; mp.fb_count = L.counters;
        k_search_merge<<<(unsigned)nq, MT, 0, st>>>(mp);
        nl += 3;
    }
    int hc[4] = {0, 0, 0, 0};
    int range_bad = 0;
    cudaMemcpyAsync(hc, L.counters, sizeof(hc), cudaMemcpyDeviceToHost, st);
    cudaMemcpyAsync(&range_bad, &qs->range_bad, sizeof(int), cudaMemcpyDeviceToHost, st);
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) { err = cudaGetErrorString(e); return SLX_ECUDA; }
    if (range_bad) { err = "lattice query: a quantized component does not fit 32 bits"; return SLX_ERANGE; }
    if (hc[2] & KERR_TIMEOUT) { err = "lattice query: tensor-core pass timed out"; return SLX_ETIMEOUT; }
    const int nfb = exact_only ? nq : hc[0];
    if (n_fallback) *n_fallback = nfb;
    if (nfb > 0) {
        const int64_t want = std::max<int64_t>(1, (2 * 148 + nfb - 1) / nfb);
        const int64_t xchunks = std::max<int64_t>(1, std::min<int64_t>(want, (L.n + 2047) / 2048));
        const int64_t rows_per = (L.n + xchunks - 1) / xchunks;
        const int xslots = (int)xchunks * (EXACT_THREADS / 32);
        const size_t xneed = (size_t)nfb * xslots * T * 12 + 1024;
        if (xneed > L.xws_bytes) {
            cudaFree(L.xws);
            L.xws = nullptr;
            L.xws_bytes = 0;
            if (cudaMalloc(&L.xws, xneed) != cudaSuccess) { cudaGetLastError(); err = "lattice query: scratch"; return SLX_EOOM; }
            L.xws_bytes = xneed;
        }
        uint8_t* xc = (uint8_t*)L.xws;
        int64_t* xkey = carve<int64_t>(xc, (size_t)nfb * xslots * T);
        int32_t* xid = carve<int32_t>(xc, (size_t)nfb * xslots * T);
        const int* ql = exact_only ? nullptr : fb_list;
        const size_t xsmem = (size_t)dim * 4;
        slx::ensure_smem((const void*)k_search_exact, xsmem);
        k_search_exact<<<dim3((unsigned)xchunks, (unsigned)nfb), EXACT_THREADS, xsmem, st>>>(
            L.vals, L.n, dim, qvals, ql, rows_per, xslots, xkey, xid);
        MergeParams mp{};
        mp.nslots = xslots; mp.k = k; mp.mode = 1; mp.ckey = xkey; mp.cid = xid; mp.qlist = ql;
        mp.n = L.n; mp.id_base = L.id_base; mp.out_ids = d_ids; mp.out_dist = d_dist; mp.payload = L.payload;
        k_search_merge<<<(unsigned)nfb, MT, 0, st>>>(mp);
        nl += 2;
    }
    if (launches) *launches += nl;
    e = cudaGetLastError();
    if (e != cudaSuccess) { err = cudaGetErrorString(e); return SLX_ECUDA; }
    return SLX_OK;
}

void merge_parts(const int64_t* ids, const uint64_t* dist, int parts, int nq, int k, int64_t* out_ids, uint64_t* out_dist,
                 cudaStream_t st) {
    k_merge_parts<<<(unsigned)((nq + 127) / 128), 128, 0, st>>>(ids, dist, parts, nq, k, out_ids, out_dist);
}

}  // namespace search
}  // namespace slx
