// k_gemv_tc.cu -- exact decode-shaped GEMV (M <= 8 activation rows) from packed Q4_0 / Q8_0 blocks,
// with the digit products on the tensor cores (tcgen05.mma kind::i8).
//
// IntegerMatMul.MatMul with the encoder's composite weights (Math/IntegerMatMul.cs:37-76,
// IntegerTransformerSource.Q = QuantizeFromFloat, :297-304): w = (long)(d * q * 2^s). For a finite f16
// scale d and 24 <= s <= 39 the product d*q*2^s is an integer below 2^63, so w = D * q with
// D = (long)(d * 2^s), and one block's contribution to an output is
//     sum_{k in block} a_k * w_k = D * sum_k a_k q_k.
// The activations are split into 5 balanced base-256 digits (a = sum_i a_i 256^i), and
//     P_i = sum_{k in block} q_k a_ik
// is exact in int32. One MMA per quant block computes P_i for all 128 weight rows of the CTA (M=128,
// the TMEM lanes) and all (activation row, digit) pairs (N = 5*M rounded up to 16), K = 32: the block.
// Each MMA writes its own TMEM columns; the epilogue (one thread per weight row) combines the digits,
// S = sum_i 256^i P_i, and accumulates S * D in Int128. Q4_0 nibbles enter the MMA as 0..15 and the
// offset of 8 is taken out once per block with the block's activation sum; a non-finite scale makes
// every composite of its block long.MinValue, i.e. S = sum_k a_k with D = long.MinValue.
//
// Two launches. k_gemv_digits splits the activations once per call into the MMA's operand layout
// (per 128-element unit: NMMA rows x 128 bytes, 128-byte swizzle), with the block sums, and marks
// activations that need a sixth digit. k_gemv_tc then streams the weights: 128 rows x 8 raw blocks
// per TMA stage (2D map over the packed rows, no multicast) into a deep ring; the CTA's slice of
// digit tiles arrives by one bulk copy; one thread per weight row unpacks 4 blocks at a time into a
// swizzled K-major tile for the MMA and runs the epilogue a few units behind. Split-K partial sums
// (Int128) are added by the last CTA of each row tile. If an activation needs a sixth digit, every
// CTA computes its part with Int128 multiply-adds of the composites instead. Every mbarrier wait is
// bounded.
#include <cuda.h>

#include <algorithm>
#include <cmath>
#include <cstring>

#include "slx_attr.h"
#include "slx_device.cuh"
#include "slx_gemm.h"
#include "slx_kernels.h"
#include "tc_ptx.cuh"

namespace slx {
namespace {

using namespace tc;

// Warps: 0 TMA, 1 TMEM + MMA, then the converters (8 for M <= 4: one group of 4 per unit of a stage;
// else 4 for both units), then 4 epilogue warps (one per TMEM lane quadrant).
__host__ __device__ constexpr int conv_warps(int m) { return m <= 4 ? 8 : 4; }
__host__ __device__ constexpr int threads_of(int m) { return 32 * (2 + conv_warps(m) + 4); }
constexpr int ROWS = 128;        // weight rows per CTA
constexpr int CB = 8;            // quant blocks per TMA stage (256 elements)
constexpr int ND = 5;            // activation digits
constexpr int FLAG_WORD = 16;    // int index of the overflow word in the workspace
constexpr size_t SMEM_CAP = 220 * 1024;

__host__ __device__ constexpr int nmma_of(int m) { return ((ND * m + 15) / 16) * 16; }
__host__ __device__ constexpr int unit_bytes(int m) { return nmma_of(m) * 128; }
// The pipeline moves in stages of 8 blocks (two 4-block units), with two rings of stage slots.
// Weight tiles (2 x 16 KB per slot): a slot is free once the MMAs of its stage have read it.
// Accumulators (8 x NMMA TMEM columns per slot) and block scales: a slot is free once the epilogue is
// done with it, so the epilogue can trail the MMAs by up to tslots_of stages. (Barrier polls cost the
// MMA thread about as much as an MMA, so they are taken once per stage.)
__host__ __device__ constexpr int tslots_of(int m) { return 512 / (8 * nmma_of(m)) >= 4 ? 4 : 512 / (8 * nmma_of(m)) >= 2 ? 2 : 1; }
__host__ __device__ constexpr int aslots_of(int m) { return tslots_of(m) < 2 ? tslots_of(m) : 2; }
__host__ __device__ constexpr int tcols_of(int m) {
    return tslots_of(m) * 8 * nmma_of(m) <= 128 ? 128 : tslots_of(m) * 8 * nmma_of(m) <= 256 ? 256 : 512;
}
__host__ __device__ constexpr int raw_bytes(bool q4) { return ROWS * CB * (q4 ? 18 : 34); }
// a TMA stage: 128 rows x 8 raw blocks, then the two units' activation digit tiles
__host__ __device__ constexpr int stage_bytes(bool q4, int m) { return raw_bytes(q4) + 2 * unit_bytes(m); }
constexpr int MAXCH = 32;  // 256-element chunks per CTA (bounds the block sums kept in shared memory)
__host__ __device__ constexpr size_t fixed_smem(int m) {
    return 1024 + (size_t)aslots_of(m) * 2 * ROWS * 128 + (size_t)tslots_of(m) * 8 * ROWS * 2 + (size_t)2 * MAXCH * m * 32 + 512;
}
// ring depth: as many stages as fit beside the rest (one CTA per SM), at most 8; the weight stream
// needs about 150 KB in flight per SM to cover the loaded TMA latency
__host__ __device__ constexpr int stages_of(bool q4, int m) {
    return (int)((SMEM_CAP - fixed_smem(m)) / stage_bytes(q4, m)) > 8 ? 8 : (int)((SMEM_CAP - fixed_smem(m)) / stage_bytes(q4, m));
}
__host__ __device__ constexpr size_t smem_bytes(bool q4, int m) {
    return fixed_smem(m) + (size_t)stages_of(q4, m) * stage_bytes(q4, m);
}

// Activations representable in 5 balanced base-256 digits.
constexpr int64_t DIG5_MAX = 0x7F7F7F7F7FLL, DIG5_MIN = -0x8080808080LL;

// Digit tiles: dig[unit][NMMA rows][128 B] with row j = m*5 + i (rows from 5*M on are zero) and the
// 16-byte chunk g of row j at position g ^ (j & 7) (the MMA's 128-byte swizzle); asum[unit][m][4].
// Per unit, threads rem < 8*M split activation row m's 16-element group g; the rest clear pad chunks.
// It also clears the split-K counters of the GEMV that follows (the workspace is shared with other
// kernels, so they are set here rather than kept).
// For Q4_0 the digits of a block's 32 elements are stored in the order the unpacked nibble words give
// (per 4-byte word j of nibbles: elements 8j, 8j+2, 8j+4, 8j+6, then 8j+1, ..., 8j+7); Q8_0 keeps
// the element order.
template <bool Q4>
__global__ void k_gemv_digits(const int64_t* __restrict__ A, int64_t lda, int M, int K, int nmma,
                              uint8_t* __restrict__ dig, int64_t* __restrict__ asum, int* overflow, int tag,
                              int* __restrict__ counters, int tiles) {
    const int units = K / 128;
    const int per_unit = nmma * 8;  // threads per unit (a multiple of 8)
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t < tiles) counters[t] = 0;
    int64_t sum = 0;
    bool live = false;
    int u = 0, m = 0, g = 0;
    if (t < units * per_unit) {
        u = t / per_unit;
        const int rem = t % per_unit;
        uint8_t* tile = dig + (size_t)u * nmma * 128;
        if (rem < 8 * M) {
            live = true;
            m = rem >> 3;
            g = rem & 7;
            const int64_t* a = A + (int64_t)m * lda + u * 128 + g * 16;
            uint32_t w[ND][4];
#pragma unroll
            for (int i = 0; i < ND; i++)
#pragma unroll
                for (int q = 0; q < 4; q++) w[i][q] = 0;
            bool bad = false;
#pragma unroll
            for (int e = 0; e < 16; e++) {
                int64_t x = a[e];
                sum = wadd(sum, x);
                bad |= x > DIG5_MAX || x < DIG5_MIN;
                // byte position of element e of this 16-element group (half a block)
                const int pos = Q4 ? ((e >> 3) << 3) + ((e & 1) << 2) + ((e & 7) >> 1) : e;
#pragma unroll
                for (int i = 0; i < ND; i++) {
                    const int d = (int)(((uint64_t)x + 128u) & 255u) - 128;
                    x = (x - d) >> 8;
                    w[i][pos >> 2] |= (uint32_t)(uint8_t)(int8_t)d << (8 * (pos & 3));
                }
            }
#pragma unroll
            for (int i = 0; i < ND; i++) {
                const int j = m * ND + i;
                *(uint4*)(tile + (j >> 3) * 1024 + (j & 7) * 128 + ((g ^ (j & 7)) << 4)) =
                    make_uint4(w[i][0], w[i][1], w[i][2], w[i][3]);
            }
            if (bad) atomicExch(overflow, tag);
        } else {
            const int pr = rem - 8 * M;       // pad chunk index
            const int j = ND * M + pr / 8;    // pad row
            if (j < nmma) *(uint4*)(tile + (j >> 3) * 1024 + (j & 7) * 128 + (pr % 8) * 16) = make_uint4(0, 0, 0, 0);
        }
    }
    // a block is two groups, held by threads t and t ^ 1 of one warp
    sum = wadd(sum, (int64_t)__shfl_xor_sync(0xffffffffu, (long long)sum, 1));
    if (live && (g & 1) == 0) asum[((size_t)u * M + m) * 4 + (g >> 1)] = sum;
}

struct GtParams {
    int N, K, chunks_total, ks_count;
    const uint8_t* W;  // packed blocks (the Int128 path reads them directly)
    const int64_t* A;
    int64_t lda;
    const uint8_t* dig;    // digit tiles [unit][NMMA x 128]
    const int64_t* asum;   // [unit][M][4]
    const int* overflow;   // == tag: an activation needs a sixth digit
    int tag;
    double scale;
    int shift;
    int64_t* C;
    int64_t ldc;
    u128* partial;  // [ks][M][N]
    int* counters;  // [row tiles], cleared by k_gemv_digits
    int* err;
};

// The block's 8 words from the unit's raw words r (4 blocks of BB bytes starting 4-byte aligned):
// even blocks start on a word, odd blocks 2 bytes past one.
template <bool Q4, int BLK>
SLX_DEV uint16_t block_words(const uint32_t* r, uint32_t (&w)[8]) {
    constexpr int BB = Q4 ? 18 : 34;
    constexpr int O = BB * BLK;
    constexpr int NW = Q4 ? 4 : 8;  // payload words
    uint16_t scale;
    uint32_t x[8];
    if (O % 4 == 0) {
        scale = (uint16_t)(r[O / 4] & 0xFFFFu);
#pragma unroll
        for (int j = 0; j < NW; j++) x[j] = __funnelshift_r(r[O / 4 + j], r[O / 4 + j + 1], 16);
    } else {
        scale = (uint16_t)(r[(O - 2) / 4] >> 16);
#pragma unroll
        for (int j = 0; j < NW; j++) x[j] = r[(O + 2) / 4 + j];
    }
    if (Q4) {
        // nibble word j: low nibbles are elements 8j, 8j+2, 8j+4, 8j+6, high nibbles 8j+1, ..., 8j+7;
        // the activation digits are stored in this order
#pragma unroll
        for (int j = 0; j < 4; j++) {
            w[2 * j] = x[j] & 0x0F0F0F0Fu;
            w[2 * j + 1] = (x[j] >> 4) & 0x0F0F0F0Fu;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; j++) w[j] = x[j];
    }
    return scale;
}

// Unpacks block BLK of a unit into the row's swizzled tile row; returns the block's f16 scale bits.
template <bool Q4, int BLK>
SLX_DEV uint16_t convert_block(const uint32_t* r, uint8_t* dst_row, int sw) {
    uint32_t w[8];
    const uint16_t sb = block_words<Q4, BLK>(r, w);
    *(uint4*)(dst_row + (((2 * BLK) ^ sw) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
    *(uint4*)(dst_row + (((2 * BLK + 1) ^ sw) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
    return sb;
}

template <bool Q4, int MM>
__global__ void __launch_bounds__(threads_of(MM), 1) k_gemv_tc(const __grid_constant__ CUtensorMap tmW, GtParams p) {
    constexpr int NMMA = nmma_of(MM);
    constexpr int BB = Q4 ? 18 : 34;
    constexpr int ROWB = CB * BB;  // raw bytes of one row in a stage
    constexpr int RS = stages_of(Q4, MM);
    constexpr int RAW_B = raw_bytes(Q4);
    constexpr int STAGE_B = stage_bytes(Q4, MM);
    constexpr int ABUF = ROWS * 128;
    constexpr int UNIT_B = unit_bytes(MM);
    constexpr int TCOLS = tcols_of(MM);
    constexpr int DCA = aslots_of(MM), DC = tslots_of(MM);
    constexpr uint32_t IDESC = idesc_i8(NMMA);
    constexpr int UW = (4 * BB) / 4;  // raw words of one unit (4 blocks)
    constexpr int NCONV = conv_warps(MM);
    constexpr int EPI0 = 2 + NCONV;   // first epilogue warp
    static_assert(RS >= 2, "at least two TMA stages");
    static_assert(RAW_B % 1024 == 0 && UNIT_B % 1024 == 0, "tiles keep 1024-byte alignment");
    static_assert(DC * 8 * NMMA <= TCOLS && TCOLS <= 512, "every stage's accumulators lie inside the TMEM allocation");
    static_assert(DCA <= DC, "a weight-tile slot is reused no later than its accumulator slot");

    const int tile = blockIdx.x, ks = blockIdx.y;
    const int n0 = tile * ROWS;
    const int c0 = (int)((int64_t)ks * p.chunks_total / p.ks_count);
    const int c1 = (int)((int64_t)(ks + 1) * p.chunks_total / p.ks_count);
    const int nch = c1 - c0, nu = 2 * nch;
    const int kbase = c0 * 256;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* abuf = smem;                                  // [DCA][2][ROWS x 128 B] weights, swizzled
    uint8_t* raw = abuf + DCA * 2 * ABUF;                  // [RS] stages: [ROWS][ROWB] raw, then 2 digit tiles
    uint16_t* dsc = (uint16_t*)(raw + RS * STAGE_B);       // [DC][8][ROWS] f16 block scales
    int64_t* asum = (int64_t*)(dsc + DC * 8 * ROWS);       // [nu][MM][4] block sums of the K range
    uint64_t* bars = (uint64_t*)(asum + 2 * MAXCH * MM * 4);
    const uint32_t raw_full = smem_u32(bars), raw_empty = raw_full + 8 * RS;
    // per accumulator slot (stage % DC): a_ready (weight tiles and scales written), mma_done, tmem_free
    const uint32_t a_ready = raw_empty + 8 * RS, mma_done = a_ready + 8 * DC, tmem_free = mma_done + 8 * DC;
    const uint32_t asum_full = tmem_free + 8 * DC;
    uint32_t* tmem_slot = (uint32_t*)(bars + 2 * RS + 3 * DC + 1);
    __shared__ int s_fail, s_last;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool over = *(volatile const int*)p.overflow == p.tag;
    if (threadIdx.x == 0) {
        s_fail = 0;
        for (int i = 0; i < RS; i++) {
            mbar_init(raw_full + 8 * i, 1);
            mbar_init(raw_empty + 8 * i, NCONV + 1);  // the converter warps + the MMAs reading the digits
        }
        for (int b = 0; b < DC; b++) {
            mbar_init(a_ready + 8 * b, NCONV);
            mbar_init(mma_done + 8 * b, 1);
            mbar_init(tmem_free + 8 * b, 4);
        }
        mbar_init(asum_full, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        if (!over) {  // the block sums of this CTA's K range, one bulk copy
            mbar_expect_tx(asum_full, (uint32_t)nu * MM * 32);
            bulk_load(smem_u32(asum), p.asum + (size_t)2 * c0 * MM * 4, (uint32_t)nu * MM * 32, asum_full);
        }
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "n"(TCOLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    u128 acc[MM];
#pragma unroll
    for (int m = 0; m < MM; m++) acc[m] = 0;
    const int r = 32 * (warp & 3) + lane;  // weight row of a converter / epilogue thread (its TMEM lane)
    const int n = n0 + r;

    if (over) {  // an activation needs a sixth digit: Int128 multiply-add of the composites
        if (warp >= EPI0 && n < p.N) {
            const int64_t nblocks = (int64_t)p.N * p.K / 32;
            for (int k = kbase; k < kbase + nch * 256; k++) {
                const int64_t wq = composite(dequant_elem(Q4 ? DT_Q4_0 : DT_Q8_0, p.W, (int64_t)n * p.K + k, nblocks), 0, p.scale);
#pragma unroll
                for (int m = 0; m < MM; m++) acc[m] += (u128)((i128)p.A[(int64_t)m * p.lda + k] * wq);
            }
        }
    } else if (warp == 0) {
        if (lane == 0) {  // TMA producer: 128 rows x 8 blocks per stage
            int issued = 0;
            for (int ch = 0; ch < nch; ch++) {
                const int s = ch % RS;
                if (!mbar_wait(raw_empty + 8 * s, (uint32_t)((ch / RS) & 1) ^ 1u)) { s_fail = 1; break; }
                if (*(volatile int*)&s_fail) break;
                mbar_expect_tx(raw_full + 8 * s, STAGE_B);
                tma_load_2d(smem_u32(raw + s * STAGE_B), &tmW, (c0 + ch) * (ROWB / 2), n0, raw_full + 8 * s);
                bulk_load(smem_u32(raw + s * STAGE_B + RAW_B), p.dig + (size_t)2 * (c0 + ch) * UNIT_B, 2 * UNIT_B,
                          raw_full + 8 * s);
                issued = ch + 1;
            }
            if (*(volatile int*)&s_fail) {  // let copies still in flight land before the CTA exits
                for (int ch = issued - RS < 0 ? 0 : issued - RS; ch < issued; ch++)
                    mbar_wait(raw_full + 8 * (ch % RS), (uint32_t)(ch / RS) & 1u);
                mbar_wait(asum_full, 0);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer: one MMA per quant block into its own TMEM columns
            const uint32_t a0 = smem_u32(abuf), r0 = smem_u32(raw);
            for (int ch = 0; ch < nch; ch++) {
                const int c = ch % DC, ca = ch % DCA, s = ch % RS;
                const uint32_t ph = (uint32_t)(ch / DC) & 1u;
                // the stage's digit tiles (raw_full), its weight tiles (a_ready), a free accumulator slot
                if (!mbar_wait(raw_full + 8 * s, (uint32_t)(ch / RS) & 1u)) { s_fail = 1; break; }
                if (!mbar_wait(a_ready + 8 * c, ph)) { s_fail = 1; break; }
                if (!mbar_wait(tmem_free + 8 * c, ph ^ 1u)) { s_fail = 1; break; }
                fence_after();
                const uint32_t dt = r0 + s * STAGE_B + RAW_B;
#pragma unroll
                for (int j = 0; j < 2; j++)
#pragma unroll
                    for (int blk = 0; blk < 4; blk++)
                        umma_i8(tmem + (uint32_t)(c * 8 + j * 4 + blk) * NMMA,
                                sw128_desc(a0 + (ca * 2 + j) * ABUF + blk * 32), sw128_desc(dt + j * UNIT_B + blk * 32),
                                IDESC, 0u);
                umma_commit(mma_done + 8 * c);
                umma_commit(raw_empty + 8 * s);  // the stage's digits are read
            }
        }
    } else if (warp < EPI0) {  // converters: unpack a stage's two units into the MMA's swizzled tiles
        const int sw = r & 7;
        uint8_t* arow0 = abuf + (r >> 3) * 1024 + (r & 7) * 128;
        // with 8 converter warps, group g converts unit g of each stage; with 4, each warp converts both
        constexpr int UPW = NCONV == 8 ? 1 : 2;  // units per warp per stage
        const int g0 = NCONV == 8 ? (warp - 2) >> 2 : 0;
        bool ok = true;
        for (int ch = 0; ch < nch && ok; ch++) {
            const int s = ch % RS, c = ch % DC, ca = ch % DCA;
            if (!mbar_wait(raw_full + 8 * s, (uint32_t)(ch / RS) & 1u)) ok = false;
            // the MMAs of stage ch - DCA have read this weight-tile slot
            if (ok && ch >= DCA) ok = mbar_wait(mma_done + 8 * ((ch - DCA) % DC), (uint32_t)((ch - DCA) / DC) & 1u);
            // the epilogue is done with stage ch - DC, whose scale slot this stage reuses
            if (ok && ch >= DC) ok = mbar_wait(tmem_free + 8 * c, (uint32_t)((ch / DC) - 1) & 1u);
            if (!__all_sync(0xffffffffu, ok)) { ok = false; s_fail = 1; break; }
            // rows are an odd number of 16-byte granules (9 or 17), so 16-byte loads of consecutive rows
            // fall in distinct bank groups; a group's unit starts g0 * 4 * BB bytes in, i.e. 2 words
            // past granule G0 when that is not a granule boundary
            const uint8_t* rowp = raw + s * STAGE_B + r * ROWB;
            constexpr int NG = (UPW * 4 * BB + 8 + 15) / 16;  // granules covering the group's units
            uint32_t rg[NG * 4];
            const int G0 = (g0 * 4 * BB) >> 4;
#pragma unroll
            for (int i = 0; i < NG; i++) {
                if (G0 + i < ROWB / 16) {
                    const uint4 v4 = *(const uint4*)(rowp + (G0 + i) * 16);
                    rg[4 * i] = v4.x; rg[4 * i + 1] = v4.y; rg[4 * i + 2] = v4.z; rg[4 * i + 3] = v4.w;
                } else {
                    rg[4 * i] = rg[4 * i + 1] = rg[4 * i + 2] = rg[4 * i + 3] = 0;
                }
            }
            uint32_t rw[UPW * UW];
            if (((g0 * 4 * BB) & 15) == 0) {
#pragma unroll
                for (int i = 0; i < UPW * UW; i++) rw[i] = rg[i];
            } else {  // the second group's unit starts 8 bytes into its first granule
#pragma unroll
                for (int i = 0; i < UPW * UW; i++) rw[i] = rg[i + 2];
            }
#pragma unroll
            for (int k = 0; k < UPW; k++) {
                const int j = g0 + k;  // unit within the stage
                uint8_t* dst = arow0 + (ca * 2 + j) * ABUF;
                uint16_t* q = dsc + (c * 8 + j * 4) * ROWS + r;
                q[0] = convert_block<Q4, 0>(rw + k * UW, dst, sw);
                q[ROWS] = convert_block<Q4, 1>(rw + k * UW, dst, sw);
                q[2 * ROWS] = convert_block<Q4, 2>(rw + k * UW, dst, sw);
                q[3 * ROWS] = convert_block<Q4, 3>(rw + k * UW, dst, sw);
            }
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(a_ready + 8 * c);
                mbar_arrive(raw_empty + 8 * s);  // the warp's rows of this stage are read
            }
        }
    } else {  // epilogue: TMEM digit sums -> Int128 accumulators
        const uint32_t taddr = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
        bool ok = __all_sync(0xffffffffu, mbar_wait(asum_full, 0));
        if (!ok) s_fail = 1;
        for (int ch = 0; ch < nch && ok; ch++) {
            const int c = ch % DC;
            const uint32_t ph = (uint32_t)(ch / DC) & 1u;
            // a_ready orders the converters' scale bits before this thread's reads
            if (!__all_sync(0xffffffffu, mbar_wait(a_ready + 8 * c, ph) && mbar_wait(mma_done + 8 * c, ph))) {
                ok = false;
                s_fail = 1;
                break;
            }
            fence_after();
            const uint16_t* dq = dsc + c * 8 * ROWS + r;
#pragma unroll 1
            for (int jb = 0; jb < 8; jb++) {  // unit jb / 4, block jb % 4
                uint32_t val[NMMA];
#pragma unroll
                for (int q = 0; q < NMMA / 16; q++)
                    tmem_ld16(taddr + (uint32_t)(c * 8 + jb) * NMMA + 16 * q, *(uint32_t(*)[16])(val + 16 * q));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                // D = d * 2^s, an integer below 2^63 for a finite d when 24 <= s <= 39;
                // long.MinValue marks a non-finite scale
                const float d = h2f(dq[jb * ROWS]);
                const int64_t D = isfinite(d) ? (int64_t)((double)d * p.scale) : INT64_MIN;
                const int64_t* as_p = asum + (size_t)(2 * ch + (jb >> 2)) * MM * 4 + (jb & 3);
#pragma unroll
                for (int m = 0; m < MM; m++) {
                    const int p0 = (int)val[m * ND], p1 = (int)val[m * ND + 1], p2 = (int)val[m * ND + 2];
                    const int p3 = (int)val[m * ND + 3], p4 = (int)val[m * ND + 4];
                    const int t01 = p1 * 256 + p0, t23 = p3 * 256 + p2;  // |p_i| < 2^20
                    int64_t S = (int64_t)t01 + (int64_t)t23 * 65536 + ((int64_t)p4 << 32);
                    const int64_t as = as_p[m * 4];
                    if (Q4) S -= 8 * as;          // nibble q - 8
                    if (D == INT64_MIN) S = as;   // every composite of the block is long.MinValue
                    const uint64_t lo = (uint64_t)S * (uint64_t)D;
                    const int64_t hi = __mul64hi(S, D);
                    acc[m] += ((u128)(uint64_t)hi << 64) | lo;
                }
            }
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tmem_free + 8 * c);
        }
    }

    // outputs: the row's sums, directly or through the split-K partials of the row tile
    if (warp >= EPI0 && n < p.N) {
        if (p.ks_count == 1) {
#pragma unroll
            for (int m = 0; m < MM; m++)
                p.C[(int64_t)m * p.ldc + n] = p.shift > 0 ? lo64(sar128((i128)acc[m], p.shift)) : lo64((i128)acc[m]);
        } else {
#pragma unroll
            for (int m = 0; m < MM; m++) p.partial[((size_t)ks * MM + m) * p.N + n] = acc[m];
        }
    }
    if (p.ks_count > 1) {
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) s_last = atomicAdd(p.counters + tile, 1) == p.ks_count - 1;
        __syncthreads();
        if (s_last) {
            __threadfence();
            if (warp >= EPI0 && n < p.N) {
#pragma unroll
                for (int m = 0; m < MM; m++) {
                    u128 tt = 0;
                    for (int k2 = 0; k2 < p.ks_count; k2++) {
                        const ulonglong2 v2 = __ldcg((const ulonglong2*)(p.partial + ((size_t)k2 * MM + m) * p.N + n));
                        tt += ((u128)v2.y << 64) | v2.x;
                    }
                    p.C[(int64_t)m * p.ldc + n] = p.shift > 0 ? lo64(sar128((i128)tt, p.shift)) : lo64((i128)tt);
                }
            }
            if (threadIdx.x == 0) p.counters[tile] = 0;
        }
    }
    fence_before();
    __syncthreads();
    if (s_fail && threadIdx.x == 0 && p.err) atomicOr(p.err, KERR_TIMEOUT);
    if (warp == 1) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(TCOLS));
    }
}

// ---- host ----

int sm_count() { return slx::device_sm_count(); }

// K split (one CTA per SM): minimizes (waves) x (a CTA's chunks x a per-chunk time that grows with M,
// plus a fixed start-up and drain of about 2.5 us).
int plan_ks(int N, int K, int M) {
    // (a CTA takes at most MAXCH chunks)
    const int tiles = (N + ROWS - 1) / ROWS, chunks = K / 256, sms = sm_count();
    const double per_chunk_us = 0.35 * M, fixed_us = 2.5;
    int best = chunks;
    double best_cost = 1e300;
    for (int ks = (chunks + MAXCH - 1) / MAXCH; ks <= chunks; ks++) {
        const double cost = std::ceil((double)tiles * ks / sms) * ((chunks + ks - 1) / ks * per_chunk_us + fixed_us);
        if (cost < best_cost - 1e-9) { best_cost = cost; best = ks; }
    }
    return best;
}

// Workspace: [0, 256) flag words, row-tile counters (cleared by k_gemv_digits), split-K partials,
// digit tiles, block sums.
size_t counters_bytes(int N) { return (((size_t)(N + ROWS - 1) / ROWS) * 4 + 255) & ~(size_t)255; }
size_t partial_bytes(int M, int N, int K) { return ((size_t)K / 256 * M * (size_t)N * sizeof(u128) + 255) & ~(size_t)255; }
size_t digit_bytes(int M, int K) { return ((size_t)K / 128 * unit_bytes(M) + 255) & ~(size_t)255; }

template <bool Q4, int MM>
void launch_tc(const WDesc& w, const int64_t* a, int64_t lda, int64_t* c, int64_t ldc, int shift, GemmWorkspace& ws,
               cudaStream_t st) {
    const int N = (int)w.N, K = (int)w.K;
    constexpr size_t smem = smem_bytes(Q4, MM);
    slx::ensure_smem((const void*)k_gemv_tc<Q4, MM>, smem);
    uint8_t* base = (uint8_t*)ws.p;
    int* flag = (int*)base + FLAG_WORD;
    int* counters = (int*)(base + 256);
    u128* partial = (u128*)(base + 256 + counters_bytes(N));
    uint8_t* dig = (uint8_t*)partial + partial_bytes(MM, N, K);
    int64_t* asum = (int64_t*)(dig + digit_bytes(MM, K));
    ws.tag = ws.tag >= 0x3fffffffu ? 1u : ws.tag + 1u;  // never 0, the cleared value
    const int tiles = (N + ROWS - 1) / ROWS;
    const int threads = std::max(K / 128 * nmma_of(MM) * 8, tiles);
    k_gemv_digits<Q4><<<(threads + 255) / 256, 256, 0, st>>>(a, lda, MM, K, nmma_of(MM), dig, asum, flag, (int)ws.tag,
                                                          counters, tiles);

    const int ks = plan_ks(N, K, MM);
    alignas(64) unsigned char map[128];
    const int bb = Q4 ? 18 : 34;
    tc::encode_rows_u16(map, w.data, (int64_t)(K / 32) * bb / 2, N, CB * bb / 2, ROWS);
    CUtensorMap tm;
    memcpy(&tm, map, sizeof(tm));
    GtParams p;
    p.N = N; p.K = K; p.chunks_total = K / 256; p.ks_count = ks;
    p.W = w.data; p.A = a; p.lda = lda; p.dig = dig; p.asum = asum; p.overflow = flag; p.tag = (int)ws.tag;
    p.scale = w.scale; p.shift = shift; p.C = c; p.ldc = ldc;
    p.partial = partial; p.counters = counters; p.err = ws.err;
    dim3 grid((unsigned)((N + ROWS - 1) / ROWS), (unsigned)ks);
    k_gemv_tc<Q4, MM><<<grid, threads_of(MM), smem, st>>>(tm, p);
}

template <bool Q4>
void launch_m(int M, const WDesc& w, const int64_t* a, int64_t lda, int64_t* c, int64_t ldc, int shift,
              GemmWorkspace& ws, cudaStream_t st) {
#define SLX_GT(MM) launch_tc<Q4, MM>(w, a, lda, c, ldc, shift, ws, st)
    switch (M) {
        case 1: SLX_GT(1); break;
        case 2: SLX_GT(2); break;
        case 3: SLX_GT(3); break;
        case 4: SLX_GT(4); break;
        case 5: SLX_GT(5); break;
        case 6: SLX_GT(6); break;
        case 7: SLX_GT(7); break;
        default: SLX_GT(8); break;
    }
#undef SLX_GT
}

// ---- M = 1: digit products on the CUDA cores (dp4a) --------------------------------------------
// For one activation row a tensor-core tile is mostly padding and every quant block needs
// its own trip through TMEM (its scale differs), so these shapes run on the CUDA cores: each lane
// holds one block's activation digits (5 digits x 8 words per row) in registers and reuses them for
// R weight rows; per (row, block) the weights are 8 words of int8x4 (Q4_0 nibbles 0..15, Q8_0
// bytes), P_i = sum dp4a(weights, digit i) is exact in int32, S = sum_i 256^i P_i, and S * D is
// added in Int128 exactly as the tensor-core kernel's epilogue does. Lanes stride the blocks of a
// row and reduce their Int128 sums at the end. (An fp64 variant, S = sum a_k q_k by DFMA, exact for
// these ranges, measured slower on this part: 25.5 / 29.8 us against 18.4 / 20.3 us.)

// dig[m][digit][word][b] (consecutive blocks adjacent, so a warp's lanes read one coalesced line per
// word) in the weight words' element order (as block_words unpacks them), asum[m][b] = sum of the
// block's activations, and the overflow tag when a value needs a sixth digit.
template <bool Q4>
__global__ void k_gemv_digits_lin(const int64_t* __restrict__ A, int64_t lda, int M, int nb,
                                  uint32_t* __restrict__ dig, int64_t* __restrict__ asum, int* overflow, int tag) {
    // four threads per block, thread q of a block taking elements 8q .. 8q+7 (payload words 2q, 2q+1
    // in both formats); the block sum is reduced over the four lanes
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    const bool live = t < M * nb * 4;
    const int blk = t >> 2, q = t & 3;
    const int m = live ? blk / nb : 0, b = live ? blk % nb : 0;
    uint32_t w[ND][2];
#pragma unroll
    for (int i = 0; i < ND; i++) w[i][0] = w[i][1] = 0;
    int64_t sum = 0;
    bool bad = false;
    if (live) {
        const int64_t* a = A + (int64_t)m * lda + (int64_t)b * 32 + 8 * q;
#pragma unroll
        for (int e = 0; e < 8; e++) {
            int64_t x = a[e];
            sum = wadd(sum, x);
            bad |= x > DIG5_MAX || x < DIG5_MIN;
            const int word = Q4 ? (e & 1) : e >> 2;  // of the thread's two words
            const int byte = Q4 ? e >> 1 : e & 3;
#pragma unroll
            for (int i = 0; i < ND; i++) {
                const int d = (int)(((uint64_t)x + 128u) & 255u) - 128;
                x = (x - d) >> 8;
                w[i][word] |= (uint32_t)(uint8_t)(int8_t)d << (8 * byte);
            }
        }
    }
    sum = wadd(sum, (int64_t)__shfl_xor_sync(0xffffffffu, (long long)sum, 1));
    sum = wadd(sum, (int64_t)__shfl_xor_sync(0xffffffffu, (long long)sum, 2));
    if (!live) return;
#pragma unroll
    for (int i = 0; i < ND; i++)
#pragma unroll
        for (int j = 0; j < 2; j++) dig[((size_t)(m * ND + i) * 8 + 2 * q + j) * nb + b] = w[i][j];
    if (q == 0) asum[(size_t)m * nb + b] = sum;
    if (bad) atomicExch(overflow, tag);
}

SLX_DEV int dp4a_s32(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

SLX_DEV void add128(uint64_t& lo, int64_t& hi, uint64_t l2, int64_t h2) {
    const uint64_t s = lo + l2;
    hi = (int64_t)((uint64_t)hi + (uint64_t)h2 + (s < lo ? 1u : 0u));
    lo = s;
}

struct DpParams {
    int N, K;
    const uint8_t* W;
    const int64_t* A;
    int64_t lda;
    const uint32_t* dig;
    const int64_t* asum;
    const int* overflow;
    int tag;
    double scale;
    int shift;
    int64_t* C;
    int64_t ldc;
};

constexpr int DPW = 4;  // warps per CTA

// Raw words of the block at byte offset o: NW + 1 words from o rounded down to 4 bytes (an odd block
// starts 2 bytes early, inside the previous block), and their unpacking into scale and payload.
template <bool Q4>
SLX_DEV void load_raw(const uint8_t* __restrict__ W, int64_t o, uint32_t (&v)[(Q4 ? 4 : 8) + 1]) {
    constexpr int NW = Q4 ? 4 : 8;
    const uint32_t* r = (const uint32_t*)(W + (o & ~(int64_t)3));
#pragma unroll
    for (int j = 0; j <= NW; j++) v[j] = __ldg(r + j);
}
template <bool Q4>
SLX_DEV uint16_t unpack_raw(int64_t o, const uint32_t (&v)[(Q4 ? 4 : 8) + 1], uint32_t (&w)[8]) {
    constexpr int NW = Q4 ? 4 : 8;
    uint32_t x[8];
    uint16_t scale;
    if ((o & 3) == 0) {
        scale = (uint16_t)(v[0] & 0xFFFFu);
#pragma unroll
        for (int j = 0; j < NW; j++) x[j] = __funnelshift_r(v[j], v[j + 1], 16);
    } else {
        scale = (uint16_t)(v[0] >> 16);
#pragma unroll
        for (int j = 0; j < NW; j++) x[j] = v[j + 1];
    }
    if (Q4) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            w[2 * j] = x[j] & 0x0F0F0F0Fu;
            w[2 * j + 1] = (x[j] >> 4) & 0x0F0F0F0Fu;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; j++) w[j] = x[j];
    }
    return scale;
}

SLX_DEV void gv_cp16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
SLX_DEV void gv_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
SLX_DEV void gv_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// A warp streams its R rows through shared memory: each step copies the rows' next 32 quant blocks
// (32 * BB bytes a row, 16-byte aligned since K % 256 == 0) with 16-byte cp.async, one step ahead of
// the arithmetic; each lane then reads its own block's words from shared memory.
template <bool Q4, int MM, int R>
__global__ void __launch_bounds__(DPW * 32) k_gemv_dp4a(DpParams p) {
    constexpr int BB = Q4 ? 18 : 34;
    constexpr int NV = (Q4 ? 4 : 8) + 1;
    constexpr int SEG = 32 * BB;  // bytes of one row's 32 blocks
    __shared__ __align__(16) uint8_t seg[DPW][2][R * SEG];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = p.K / 32;
    const int n0 = (blockIdx.x * DPW + warp) * R;
    if (n0 >= p.N) return;
    const bool wide = *(volatile const int*)p.overflow == p.tag;  // an activation needs a sixth digit
    const int steps = (nb + 31) / 32;
    auto issue = [&](int it, int buf) {
        const int blocks = min(32, nb - 32 * it);  // a multiple of 8: whole 16-byte chunks
        const int chunks = blocks * BB / 16;
        const uint32_t dst = (uint32_t)__cvta_generic_to_shared(seg[warp][buf]);
#pragma unroll
        for (int r = 0; r < R; r++) {
            if (n0 + r >= p.N) break;
            const uint8_t* src = p.W + ((int64_t)(n0 + r) * nb + 32 * it) * BB;
            for (int c = lane; c < chunks; c += 32) gv_cp16(dst + r * SEG + c * 16, src + c * 16);
        }
        gv_commit();
    };
    uint64_t lo[R][MM];
    int64_t hi[R][MM];
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int m = 0; m < MM; m++) lo[r][m] = 0, hi[r][m] = 0;
    issue(0, 0);
    for (int it = 0; it < steps; it++) {
        if (it + 1 < steps) {
            issue(it + 1, (it + 1) & 1);
            gv_wait<1>();
        } else {
            gv_wait<0>();
        }
        __syncwarp();
        const int b = 32 * it + lane;
        const uint8_t* sb = seg[warp][it & 1];
        if (b < nb) {
            uint32_t dq[MM][ND][8];
            int64_t as[MM];
            if (!wide) {
#pragma unroll
                for (int m = 0; m < MM; m++) {
#pragma unroll
                    for (int i = 0; i < ND; i++)
#pragma unroll
                        for (int j = 0; j < 8; j++)
                            dq[m][i][j] = __ldg(p.dig + ((size_t)(m * ND + i) * 8 + j) * nb + b);
                    as[m] = __ldg(p.asum + (size_t)m * nb + b);
                }
            }
#pragma unroll
            for (int r = 0; r < R; r++) {
                const int n = n0 + r;
                if (n >= p.N) break;
                const int64_t o = (int64_t)lane * BB;  // the block's offset in its segment (same parity as in W)
                uint32_t v[NV];
                const uint32_t* wsrc = (const uint32_t*)(sb + r * SEG + (o & ~(int64_t)3));
#pragma unroll
                for (int j = 0; j < NV; j++) v[j] = wsrc[j];
                uint32_t wq[8];
                const float d = h2f(unpack_raw<Q4>(o, v, wq));
                // D = d * 2^s (an integer below 2^63 for a finite d); long.MinValue marks a non-finite scale
                const int64_t D = isfinite(d) ? (int64_t)((double)d * p.scale) : INT64_MIN;
                if (!wide) {
#pragma unroll
                    for (int m = 0; m < MM; m++) {
                        int P[ND];
#pragma unroll
                        for (int i = 0; i < ND; i++) {
                            int acc = 0;
#pragma unroll
                            for (int j = 0; j < 8; j++) acc = dp4a_s32(wq[j], dq[m][i][j], acc);
                            P[i] = acc;
                        }
                        const int t01 = P[1] * 256 + P[0], t23 = P[3] * 256 + P[2];  // |P_i| < 2^20
                        int64_t S = (int64_t)t01 + (int64_t)t23 * 65536 + ((int64_t)P[4] << 32);
                        if (Q4) S -= 8 * as[m];
                        if (D == INT64_MIN) S = as[m];  // every composite of the block is long.MinValue
                        add128(lo[r][m], hi[r][m], (uint64_t)S * (uint64_t)D, __mul64hi(S, D));
                    }
                } else {
                    // Int128 multiply-adds of the composites w = D * q (long.MinValue for a non-finite scale)
                    for (int e = 0; e < 32; e++) {
                        const int word = Q4 ? 2 * (e >> 3) + (e & 1) : e >> 2;
                        const int byte = Q4 ? (e & 7) >> 1 : e & 3;
                        const int q = Q4 ? (int)((wq[word] >> (8 * byte)) & 15u) - 8
                                         : (int)(int8_t)(uint8_t)(wq[word] >> (8 * byte));
                        const int64_t wc = D == INT64_MIN ? INT64_MIN : D * q;
#pragma unroll
                        for (int m = 0; m < MM; m++) {
                            const int64_t x = p.A[(int64_t)m * p.lda + (int64_t)b * 32 + e];
                            add128(lo[r][m], hi[r][m], (uint64_t)x * (uint64_t)wc, __mul64hi(x, wc));
                        }
                    }
                }
            }
        }
        __syncwarp();  // every lane is done with this buffer before it is refilled
    }
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int m = 0; m < MM; m++) {
            uint64_t l = lo[r][m];
            int64_t h = hi[r][m];
            for (int o = 16; o > 0; o >>= 1) {
                const uint64_t l2 = __shfl_xor_sync(0xffffffffu, (unsigned long long)l, o);
                const int64_t h2 = __shfl_xor_sync(0xffffffffu, (long long)h, o);
                add128(l, h, l2, h2);
            }
            const int n = n0 + r;
            if (lane == 0 && n < p.N) {
                const i128 v = (i128)(((u128)(uint64_t)h << 64) | l);
                p.C[(int64_t)m * p.ldc + n] = p.shift > 0 ? lo64(sar128(v, p.shift)) : lo64(v);
            }
        }
}

template <bool Q4, int MM>
void launch_dp4a(const WDesc& w, const int64_t* a, int64_t lda, int64_t* c, int64_t ldc, int shift, GemmWorkspace& ws,
                 cudaStream_t st) {
    const int N = (int)w.N, K = (int)w.K, nb = K / 32;
    uint8_t* base = (uint8_t*)ws.p;
    int* flag = (int*)base + FLAG_WORD;
    uint8_t* dig = base + 256 + counters_bytes(N) + partial_bytes(MM, N, K);  // the digit-tile region
    int64_t* asum = (int64_t*)(dig + digit_bytes(MM, K));
    ws.tag = ws.tag >= 0x3fffffffu ? 1u : ws.tag + 1u;
    k_gemv_digits_lin<Q4><<<(MM * nb * 4 + 127) / 128, 128, 0, st>>>(a, lda, MM, nb, (uint32_t*)dig, asum, flag,
                                                                    (int)ws.tag);
    DpParams p;
    p.N = N; p.K = K; p.W = w.data; p.A = a; p.lda = lda; p.dig = (const uint32_t*)dig; p.asum = asum;
    p.overflow = flag; p.tag = (int)ws.tag; p.scale = w.scale; p.shift = shift; p.C = c; p.ldc = ldc;
    constexpr int R = 4;  // rows per warp
    k_gemv_dp4a<Q4, MM, R><<<(unsigned)((N + DPW * R - 1) / (DPW * R)), DPW * 32, 0, st>>>(p);
}

}  // namespace

bool gemv_supported(const WDesc& w, int M) {
    // d * 2^s is an integer for every f16 d only when s >= 24 (the smallest subnormal is 2^-24), and
    // d * q * 2^s stays below 2^63 for every finite d and q when s <= 39
    return M >= 1 && M <= 8 && w.mode == 0 && (w.dtype == DT_Q4_0 || w.dtype == DT_Q8_0) && w.K % 256 == 0 &&
           w.scale >= 16777216.0 && w.scale <= 549755813888.0 && w.nblocks * 32 >= w.N * w.K &&
           ((uintptr_t)w.data & 15) == 0 && w.N <= (int64_t)INT32_MAX / 2;
}

size_t gemv_workspace(int M, int N, int K) {
    return 256 + counters_bytes(N) + partial_bytes(M, N, K) + digit_bytes(M, K) + (size_t)K / 32 * M * 8 + 256;
}

bool gemv_reserve(GemmWorkspace& ws, int M, int N, int K, cudaStream_t st) {
    const size_t need = gemv_workspace(M, N, K);
    if (need <= ws.bytes) return true;
    if (ws.p) cudaFree(ws.p);
    ws.p = nullptr;
    ws.bytes = 0;
    ws.tag = 0;
    ws.gen++;
    if (cudaMalloc(&ws.p, need) != cudaSuccess) return false;
    ws.bytes = need;
    cudaMemsetAsync(ws.p, 0, need, st);  // the overflow word starts below every tag
    return true;
}

int gemv_exact(const int64_t* a, int64_t lda, int M, const WDesc& w, int64_t* c, int64_t ldc, int shift,
               GemmWorkspace& ws, cudaStream_t st) {
    if (M == 1) {
        if (gemv1(w, a, c, shift, ws.err, st)) return 1;
        if (w.dtype == DT_Q4_0) launch_dp4a<true, 1>(w, a, lda, c, ldc, shift, ws, st);
        else launch_dp4a<false, 1>(w, a, lda, c, ldc, shift, ws, st);
        return 2;
    }
    if (w.dtype == DT_Q4_0)
        launch_m<true>(M, w, a, lda, c, ldc, shift, ws, st);
    else
        launch_m<false>(M, w, a, lda, c, ldc, shift, ws, st);
    return 2;
}

}  // namespace slx
