// k_gemv1.cu -- exact single-row GEMV (M = 1) streaming packed Q4_0 / Q8_0 blocks.
//
// IntegerMatMul.MatMul (Math/IntegerMatMul.cs:37-76) for one activation row and the encoder's
// composite weights w = (long)(d * q * 2^s) = D * q (QuantizeFromFloat, :297-304; D = (long)(d * 2^s)
// is an integer for every finite f16 scale d when 24 <= s <= 39): one block's share of an output is
// D * sum_{k in block} a_k q_k. With the activations split into five balanced base-256 digits
// (a = sum_i a_i 256^i), P_i = sum_k q_k a_ik is an exact int32 dp4a chain, S = sum_i 256^i P_i, and
// S * D is added in Int128.
//
// One launch of persistent CTAs (two per SM), each owning a contiguous range of weight rows, so its
// blocks are one contiguous byte range of the weight:
//   * a producer warp streams that range in stages of SR rows with 1D bulk copies (cp.async.bulk,
//     no multicast) into a ring of NS shared-memory slots, each slot an mbarrier with a byte count;
//   * the consumers stage the activation row in shared memory with coalesced loads; every consumer
//     thread then owns one block column b of the row (K / 32 columns, in RG row groups that take
//     alternate stages) and forms that column's 40 activation digit words, once, in registers; per
//     stage it reads its block of each of the SR rows from shared memory (5 or 9 words), runs the
//     40 dp4a and the Int128 multiply-add;
//   * the SR per-row partial sums of a warp are reduced by a butterfly (SR Int128 values shrink to
//     one per lane), the group's warps leave theirs in shared memory, and the last warp of the group
//     to arrive (an atomic count, no barrier) adds them and writes lo64(sum >> shift) for the rows.
// An activation outside the five-digit range makes the CTA take Int128 multiply-adds of the
// composites instead (every CTA sees the same activations, so all of them do). Every mbarrier wait
// is bounded; on a timeout the kernel records KERR_TIMEOUT, lets its copies land and returns.
#include <cuda.h>

#include <algorithm>
#include <cmath>

#include "slx_attr.h"
#include "slx_device.cuh"
#include "slx_gemm.h"
#include "slx_kernels.h"
#include "tc_ptx.cuh"

namespace slx {
namespace {

constexpr int G1_ND = 5;      // activation digits
// weight rows per stage: 8 for Q4_0 (more rows share each stage's reduction), 4 for Q8_0 (twice the
// bytes per row; measured faster with the shorter stages)
template <bool Q4>
__host__ __device__ constexpr int g1_sr() { return Q4 ? 8 : 4; }
constexpr int G1_CONS = 256;  // consumer threads
constexpr int G1_THREADS = G1_CONS + 32;

struct G1Params {
    int N, NB;    // rows, blocks per row (K / 32)
    int stages;   // ceil(N / SR)
    int nbp, rg;  // block columns rounded to warps, row groups (rg * nbp <= 256)
    int ns;       // ring slots
    const uint8_t* W;
    const int64_t* A;
    int sbits;    // the composite scale 2^sbits (24..39)
    int shift;
    int64_t* C;
    int* err;
};

template <bool Q4>
__host__ __device__ constexpr int g1_bb() { return Q4 ? 18 : 34; }

__device__ __forceinline__ int g1_dp4a(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ void g1_add128(uint64_t& lo, int64_t& hi, uint64_t l2, int64_t h2) {
    const uint64_t s = lo + l2;
    hi = (int64_t)((uint64_t)hi + (uint64_t)h2 + (s < lo ? 1u : 0u));
    lo = s;
}

__device__ __forceinline__ void g1_bulk(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// The block at byte offset o of a stage slot: scale bits and the 8 payload words in the element
// order of the digit words (Q4_0: word 2j = low nibbles of payload bytes 4j..4j+3, word 2j+1 their high
// nibbles; Q8_0: the payload bytes in order). o is even, so the payload (byte o + 2) starts on a word
// boundary or halfway into one: one funnel shift by 0 or 16 bits per word, the same code for every lane.
template <bool Q4>
__device__ __forceinline__ uint32_t g1_block(const uint8_t* slot, int o, uint32_t (&w)[8]) {
    constexpr int NW = Q4 ? 4 : 8;
    const uint32_t* r = (const uint32_t*)(slot + ((o + 2) & ~3));
    const uint32_t sh = (uint32_t)((o + 2) & 3) * 8u;
    uint32_t v[NW + 1];
#pragma unroll
    for (int j = 0; j <= NW; j++) v[j] = r[j];
    const uint32_t scale = *(const uint16_t*)(slot + o);
    uint32_t x[NW];
#pragma unroll
    for (int j = 0; j < NW; j++) x[j] = __funnelshift_r(v[j], v[j + 1], sh);
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

// D = (long)(d * 2^sbits) for the f16 scale bits h, exactly (an integer for 24 <= sbits <= 39);
// INT64_MIN for a non-finite d (the reference's (long) of NaN / infinity on x64).
__device__ __forceinline__ int64_t g1_scale(uint32_t h, int sbits) {
    const uint32_t ex = (h >> 10) & 31u, mant = h & 1023u;
    if (ex == 31u) return INT64_MIN;
    const int64_t m = ex ? (int64_t)(mant | 1024u) : (int64_t)mant;
    const int64_t D = m << (ex ? (int)ex - 25 + sbits : sbits - 24);
    return (h & 0x8000u) ? -D : D;
}

// S * D in Int128 for a finite scale, from D = +-m 2^e (m the 11-bit significand, 0 <= e <= 44):
// the 64-bit product S m (|S m| < 2^63 for the block sums here) shifted left by e.
__device__ __forceinline__ void g1_mul_scale(int64_t S, uint32_t h, int sbits, uint64_t& lo, int64_t& hi) {
    const uint32_t ex = (h >> 10) & 31u, mant = h & 1023u;
    const int64_t m = ex ? (int64_t)(mant | 1024u) : (int64_t)mant;
    const int e = ex ? (int)ex - 25 + sbits : sbits - 24;
    const int64_t p = (h & 0x8000u) ? -(S * m) : S * m;
    lo = (uint64_t)p << e;
    hi = (p >> 1) >> (63 - e);  // the bits shifted out of the low word, sign-extended
}

// One block of one row by Int128 multiply-adds of the composites w = D * q (long.MinValue for a
// non-finite scale): the path for activations outside the five-digit range.
template <bool Q4>
__device__ __noinline__ void g1_block_wide(const uint8_t* blk, int64_t D, const int64_t* a, uint64_t& lo, int64_t& hi) {
#pragma unroll 1
    for (int e = 0; e < 32; e++) {
        const int q = Q4 ? (int)((blk[2 + (e >> 1)] >> (4 * (e & 1))) & 15u) - 8 : (int)(int8_t)blk[2 + e];
        const int64_t wc = D == INT64_MIN ? INT64_MIN : D * q;
        const int64_t x = __ldg(a + e);
        g1_add128(lo, hi, (uint64_t)x * (uint64_t)wc, __mul64hi(x, wc));
    }
}

// Butterfly reduce-scatter of KEEP Int128 values per lane across a warp: at each distance the lanes
// with that lane bit set keep the upper half of their values and the others the lower half, adding
// the partner's copy of the half they keep; once one value is left, the remaining distances sum it.
// Afterwards lane l holds, for row l / (32 / KEEP), the sum over all 32 lanes.
template <int KEEP, int N>
__device__ __forceinline__ void g1_fly(uint64_t (&lo)[N], int64_t (&hi)[N], int lane, int dist) {
    if constexpr (KEEP == 1) {
#pragma unroll
        for (int d = dist; d >= 1; d >>= 1) {
            const uint64_t ol = __shfl_xor_sync(0xffffffffu, (unsigned long long)lo[0], d);
            const int64_t oh = __shfl_xor_sync(0xffffffffu, (long long)hi[0], d);
            g1_add128(lo[0], hi[0], ol, oh);
        }
    } else {
        constexpr int H = KEEP / 2;
        const bool upper = (lane & dist) != 0;
#pragma unroll
        for (int r = 0; r < H; r++) {
            const uint64_t ol = __shfl_xor_sync(0xffffffffu, (unsigned long long)(upper ? lo[r] : lo[r + H]), dist);
            const int64_t oh = __shfl_xor_sync(0xffffffffu, (long long)(upper ? hi[r] : hi[r + H]), dist);
            if (upper) {
                lo[r] = lo[r + H];
                hi[r] = hi[r + H];
            }
            g1_add128(lo[r], hi[r], ol, oh);
        }
        g1_fly<H>(lo, hi, lane, dist >> 1);
    }
}

template <bool Q4>
__global__ void __launch_bounds__(G1_THREADS, 2) k_gemv1(G1Params p) {
    constexpr int BB = g1_bb<Q4>();
    constexpr int G1_SR = g1_sr<Q4>();
    extern __shared__ __align__(128) uint8_t g1_smem[];
    const int row_bytes = p.NB * BB;
    const int slot_bytes = G1_SR * row_bytes;
    uint64_t* bars = (uint64_t*)(g1_smem + (size_t)p.ns * slot_bytes);
    const uint32_t full0 = tc::smem_u32(bars), empty0 = tc::smem_u32(bars + p.ns);
    // per ring slot: the group's warps' Int128 row partials [slot][warp][row] and an arrival count
    uint64_t* red_lo = (uint64_t*)(bars + 2 * p.ns);
    int64_t* red_hi = (int64_t*)(red_lo + (size_t)p.ns * 8 * G1_SR);
    int* red_cnt = (int*)(red_hi + (size_t)p.ns * 8 * G1_SR);
    // the activation row, staged by coalesced loads: block b's 32 values at b * 34 (16-byte aligned rows,
    // four banks apart, so each quarter warp's 16-byte reads of 8 consecutive blocks are conflict-free)
    int64_t* as = (int64_t*)(((uintptr_t)(red_cnt + p.ns) + 15) & ~(uintptr_t)15);
    __shared__ int s_fail, s_wide;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // stages [s0, s1) of this CTA
    const int s0 = (int)((int64_t)blockIdx.x * p.stages / gridDim.x);
    const int s1 = (int)((int64_t)(blockIdx.x + 1) * p.stages / gridDim.x);
    const int nst = s1 - s0;
    const int gw = p.nbp / 32;  // warps per row group
    if (tid == 0) {
        s_fail = 0;
        s_wide = 0;
        for (int i = 0; i < p.ns; i++) {
            tc::mbar_init(full0 + 8 * i, 1);
            tc::mbar_init(empty0 + 8 * i, gw);
            red_cnt[i] = 0;
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == G1_CONS / 32) {  // producer
        if (lane == 0) {
            int issued = 0;
            bool ok = true;
            for (int i = 0; i < nst; i++) {
                const int slot = i % p.ns;
                if (!tc::mbar_wait(empty0 + 8 * slot, ((uint32_t)(i / p.ns) & 1u) ^ 1u) || *(volatile int*)&s_fail) {
                    ok = false;
                    break;
                }
                const int n0 = (s0 + i) * G1_SR;
                const int rows = min(G1_SR, p.N - n0);
                const uint32_t bytes = (uint32_t)(rows * row_bytes);
                tc::mbar_expect_tx(full0 + 8 * slot, bytes);
                g1_bulk(tc::smem_u32(g1_smem + (size_t)slot * slot_bytes), p.W + (int64_t)n0 * row_bytes, bytes,
                        full0 + 8 * slot);
                issued = i + 1;
            }
            if (!ok) {  // let copies still in flight land before the CTA exits (they always complete)
                s_fail = 1;
                for (int i = issued - p.ns < 0 ? 0 : issued - p.ns; i < issued; i++)
                    tc::mbar_wait(full0 + 8 * (i % p.ns), (uint32_t)(i / p.ns) & 1u);
            }
        }
        __syncthreads();
        if (s_fail && tid == G1_CONS && p.err) atomicOr(p.err, KERR_TIMEOUT);
        return;
    }

    // consumer thread: row group g, block column b
    const int g = tid / p.nbp, b = tid % p.nbp;
    const bool live = g < p.rg;
    const bool col = live && b < p.NB;
    // this column's activation digits: dq[j][i] = digit i of the four elements of payload word j
    uint32_t dq[8][G1_ND];
    int64_t asum = 0;
    bool wide = false;
#pragma unroll
    for (int j = 0; j < 8; j++)
#pragma unroll
        for (int i = 0; i < G1_ND; i++) dq[j][i] = 0;
    for (int i = tid; i < p.NB * 16; i += G1_CONS) {  // 16-byte granules of the row, coalesced
        const longlong2 v = __ldg((const longlong2*)p.A + i);
        *(longlong2*)(as + (i >> 4) * 34 + 2 * (i & 15)) = v;
    }
    asm volatile("bar.sync 9, %0;" ::"n"(G1_CONS) : "memory");
    if (col) {
        int64_t x[32];
#pragma unroll
        for (int e = 0; e < 16; e++) {
            const longlong2 v = *(const longlong2*)(as + b * 34 + 2 * e);
            x[2 * e] = v.x;
            x[2 * e + 1] = v.y;
        }
#pragma unroll
        for (int e = 0; e < 32; e++) asum = wadd(asum, x[e]);
        // payload word j's elements: Q4_0 word 2j' + h holds elements 8j' + h + 2t (the low / high
        // nibbles of bytes 4j'..4j'+3); Q8_0 word j holds elements 4j + t
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int e0 = Q4 ? 8 * (j >> 1) + (j & 1) : 4 * j;
            const int st = Q4 ? 2 : 1;
            digit_words4(x[e0], x[e0 + st], x[e0 + 2 * st], x[e0 + 3 * st], dq[j], wide);
        }
    }
    // CTA-wide "an activation needs a sixth digit" among the consumer threads (named barrier 9: the
    // producer warp is not part of it; every CTA sees the same activations, so all decide alike)
    if (wide) s_wide = 1;
    asm volatile("bar.sync 9, %0;" ::"n"(G1_CONS) : "memory");
    wide = *(volatile int*)&s_wide != 0;

    const int wg = (tid % p.nbp) >> 5;  // warp within the group
    for (int i = g; live && i < nst; i += p.rg) {
        const int slot = i % p.ns;
        // after a failed wait anywhere in the CTA no thread waits again (the loop runs on with zero
        // partials; the call reports the timeout)
        bool ok = *(volatile int*)&s_fail == 0;
        ok = __all_sync(0xffffffffu, ok && tc::mbar_wait(full0 + 8 * slot, (uint32_t)(i / p.ns) & 1u));
        if (!ok) s_fail = 1;
        const int n0 = (s0 + i) * G1_SR;
        const uint8_t* sl = g1_smem + (size_t)slot * slot_bytes;
        uint64_t lo[G1_SR];
        int64_t hi[G1_SR];
#pragma unroll
        for (int r = 0; r < G1_SR; r++) lo[r] = 0, hi[r] = 0;
        if (col && ok) {
#pragma unroll
            for (int r = 0; r < G1_SR; r++) {
                // rows past N (a partial last stage) compute on stale bytes of the slot; never written out
                const int o = r * row_bytes + b * BB;
                uint32_t wq[8];
                const uint32_t hs = g1_block<Q4>(sl, o, wq);
                const bool finite = ((hs >> 10) & 31u) != 31u;
                if (!wide) {
                    int P[G1_ND];
#pragma unroll
                    for (int k = 0; k < G1_ND; k++) {
                        int acc = 0;
#pragma unroll
                        for (int j = 0; j < 8; j++) acc = g1_dp4a(wq[j], dq[j][k], acc);
                        P[k] = acc;
                    }
                    const int t01 = P[1] * 256 + P[0], t23 = P[3] * 256 + P[2];  // |P_i| < 2^20
                    int64_t S = (int64_t)t01 + (int64_t)t23 * 65536 + ((int64_t)P[4] << 32);
                    if (Q4) S -= 8 * asum;
                    if (finite) {
                        g1_mul_scale(S, hs, p.sbits, lo[r], hi[r]);
                    } else {  // every composite of the block is long.MinValue: sum_k a_k * long.MinValue
                        lo[r] = (uint64_t)asum << 63;
                        hi[r] = __mul64hi(asum, INT64_MIN);
                    }
                } else {
                    g1_block_wide<Q4>(sl + o, g1_scale(hs, p.sbits), p.A + (int64_t)b * 32, lo[r], hi[r]);
                }
            }
        }
        g1_fly<G1_SR>(lo, hi, lane, 16);  // lane l: the warp's sum of row l / (32 / SR)
        constexpr int LOWB = 32 / G1_SR;  // lanes per row after the butterfly
        uint64_t* rl = red_lo + ((size_t)slot * 8 + wg) * G1_SR;
        int64_t* rh = red_hi + ((size_t)slot * 8 + wg) * G1_SR;
        if ((lane % LOWB) == 0) {
            rl[lane / LOWB] = lo[0];
            rh[lane / LOWB] = hi[0];
        }
        // the group's last warp to arrive adds the warps' partials and writes the stage's rows; the
        // slot (its bytes and partials) goes back to the producer only after that
        __threadfence_block();
        __syncwarp();
        int last = 0;
        if (lane == 0) last = atomicAdd(&red_cnt[slot], 1) == gw - 1;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence_block();
            if (lane < G1_SR && n0 + lane < p.N) {
                uint64_t l = 0;
                int64_t h = 0;
                for (int w = 0; w < gw; w++)
                    g1_add128(l, h, ((volatile uint64_t*)red_lo)[((size_t)slot * 8 + w) * G1_SR + lane],
                              ((volatile int64_t*)red_hi)[((size_t)slot * 8 + w) * G1_SR + lane]);
                const i128 v = (i128)(((u128)(uint64_t)h << 64) | l);
                p.C[n0 + lane] = p.shift > 0 ? lo64(sar128(v, p.shift)) : lo64(v);
            }
            __syncwarp();
            if (lane == 0) red_cnt[slot] = 0;
        }
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(empty0 + 8 * slot);
    }
    __syncthreads();  // pairs with the producer's
    if (s_fail && tid == 0 && p.err) atomicOr(p.err, KERR_TIMEOUT);
}

template <bool Q4>
bool launch_gemv1(const WDesc& w, const int64_t* a, int64_t* c, int shift, int* err, cudaStream_t st) {
    constexpr int BB = g1_bb<Q4>();
    constexpr int G1_SR = g1_sr<Q4>();
    const int NB = (int)(w.K / 32);
    if (NB % 8 != 0 || NB > G1_CONS || w.N <= 0 || ((uintptr_t)w.data & 15) != 0 || ((uintptr_t)a & 15) != 0)
        return false;
    int e = 0;
    if (std::frexp(w.scale, &e) != 0.5 || e - 1 < 24 || e - 1 > 39) return false;  // 2^24 .. 2^39
    G1Params p;
    p.N = (int)w.N;
    p.NB = NB;
    p.stages = (p.N + G1_SR - 1) / G1_SR;
    p.nbp = (NB + 31) / 32 * 32;
    p.rg = std::min(8, G1_CONS / p.nbp);
    const int slot = G1_SR * NB * BB;  // a multiple of 16 bytes (NB % 8 == 0)
    const size_t astage = (size_t)NB * 34 * 8 + 16;  // the staged activation row
    p.ns = (int)std::max<int64_t>(2, std::min<int64_t>(8, ((int64_t)110 * 1024 - 4096 - (int64_t)astage) / slot));
    p.W = w.data; p.A = a; p.sbits = e - 1; p.shift = shift; p.C = c; p.err = err;
    // the ring, then per slot two mbarriers, 8 warps x SR Int128 partials and a counter
    const size_t smem = (size_t)p.ns * slot + (size_t)p.ns * (16 + 8 * G1_SR * 16 + 4) + astage;
    if (smem > 112 * 1024) return false;  // two CTAs per SM
    if (slx::ensure_smem((const void*)k_gemv1<Q4>, smem) != cudaSuccess) return false;
    const int grid = std::min(2 * slx::device_sm_count(), p.stages);
    k_gemv1<Q4><<<grid, G1_THREADS, smem, st>>>(p);
    return true;
}

}  // namespace

bool gemv1(const WDesc& w, const int64_t* a, int64_t* c, int shift, int* err, cudaStream_t st) {
    if (w.dtype == DT_Q4_0) return launch_gemv1<true>(w, a, c, shift, err, st);
    if (w.dtype == DT_Q8_0) return launch_gemv1<false>(w, a, c, shift, err, st);
    return false;
}

}  // namespace slx
