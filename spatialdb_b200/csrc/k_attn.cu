// k_attn.cu -- exact integer attention with tensor-core scores.
//
// Reference semantics (Math/IntegerAttention.cs:60-109, 165-202, 246-289, 333-377), per head:
//   score[t][s] = (long)((sum_d q[t][d]*k[s][d]) >> 30) / ISqrt64(hd)   (masked slots: -2^29)
//   p[t][s]     = FixedSoftmax(score[t][:])                              (IntegerTranscendentals.cs:71-97)
//   out[t][d]   = sum_s (long)(((Int128)p[t][s] * v[s][d]) >> 30)       (floor per term, wrapping sum)
// Scores come from the tcgen05 digit GEMM (k_gemm_tc.cu, 5 x 5 balanced digits of q and k). The
// softmax and the per-term floor run here on CUDA cores: with v = v_hi*2^30 + v_lo
// (v_lo in [0, 2^30)) and 0 <= p <= 2^30,
//   floor(p*v / 2^30) = p*v_hi + floor(p*v_lo / 2^30),
// and floor(p*v_lo / 2^30) = umulhi(4p, v_lo) (+ v_lo when p == 2^30), two 32-bit multiplies a term.
// Any row outside that fast range (q/k wider than 5 digits, an exp above 2^30 after a long
// wrap-around, |v_hi| >= 2^31) raises the call's flag, and the exact kernel redoes the call.
#include "slx_device.cuh"
#include "slx_gemm.h"
#include "slx_kernels.h"

namespace slx {
namespace {

constexpr int PR = 16;   // query rows per block
constexpr int PT = 256;  // threads per block
constexpr int VT = 32;   // keys per V tile

// Division of n < 2^63 by an invariant d in [1, 2^63): floor via a 64-bit reciprocal estimate and
// a bounded correction (the estimate is at most 2 below the quotient).
SLX_DEV uint64_t udiv_inv(uint64_t n, uint64_t d, uint64_t inv) {
    uint64_t q = __umul64hi(n, inv);
    uint64_t r = n - q * d;
    while (r >= d) { q++; r -= d; }
    return q;
}

// out[t][d] = sum_s floor(p[t][s] * v[s][d] / 2^30) for the block's rows, wrapping sums.
// p * v = p * v_hi * 2^30 + p * v_lo, so each term is p*v_hi + umulhi(p, 4*v_lo) exactly.
template <int RPT, int HD>
__device__ __forceinline__ void pv_rows(const uint32_t* __restrict__ P, int Tp, const int64_t* __restrict__ vb, int64_t ldv,
                                        uint32_t* Vlo4, int32_t* Vhi, int T, int t0, int64_t* __restrict__ O, int64_t ldo,
                                        int b, int h, int* s_bad) {
    constexpr int G = PT / HD;  // row groups
    static_assert(G * RPT == PR, "rows per block");
    const int d = threadIdx.x % HD, g = threadIdx.x / HD;
    int64_t acc_hi[RPT];   // sum of p * v_hi (two's-complement wrap, as the reference's long adds)
    uint64_t acc_lo[RPT];  // sum of floor(p * v_lo / 2^30)
#pragma unroll
    for (int j = 0; j < RPT; j++) { acc_hi[j] = 0; acc_lo[j] = 0; }
    for (int s0 = 0; s0 < Tp; s0 += VT) {
        __syncthreads();
        for (int i = threadIdx.x; i < VT * HD; i += PT) {
            const int s = s0 + i / HD, dd = i % HD;
            int64_t v = s < T ? vb[(int64_t)s * ldv + dd] : 0;
            const int64_t hi = v >> 30;
            if (hi < INT32_MIN || hi > INT32_MAX) *s_bad = 1;
            Vhi[i] = (int32_t)hi;
            Vlo4[i] = (uint32_t)(v & ((1LL << 30) - 1)) << 2;
        }
        __syncthreads();
        if (*s_bad) return;
        const int nk = min(VT, Tp - s0);
        for (int s = 0; s < nk; s += 4) {
            uint32_t lo[4];
            int32_t hi[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                lo[u] = Vlo4[(s + u) * HD + d];
                hi[u] = Vhi[(s + u) * HD + d];
            }
#pragma unroll
            for (int j = 0; j < RPT; j++) {
                const uint4 p4 = *(const uint4*)(P + (size_t)(g + G * j) * Tp + s0 + s);
                int64_t ah = acc_hi[j];
                // p <= 2^30 fits s32: one mad.wide.s32 per term (64-bit wrap-around sum)
                asm("mad.wide.s32 %0, %1, %2, %0;" : "+l"(ah) : "r"((int32_t)p4.x), "r"(hi[0]));
                asm("mad.wide.s32 %0, %1, %2, %0;" : "+l"(ah) : "r"((int32_t)p4.y), "r"(hi[1]));
                asm("mad.wide.s32 %0, %1, %2, %0;" : "+l"(ah) : "r"((int32_t)p4.z), "r"(hi[2]));
                asm("mad.wide.s32 %0, %1, %2, %0;" : "+l"(ah) : "r"((int32_t)p4.w), "r"(hi[3]));
                acc_hi[j] = ah;
                // each floor(p * 4 v_lo / 2^32) < 2^30, so four of them sum below 2^32
                const uint32_t q = __umulhi(p4.x, lo[0]) + __umulhi(p4.y, lo[1]) + __umulhi(p4.z, lo[2]) +
                                   __umulhi(p4.w, lo[3]);
                acc_lo[j] += q;
            }
        }
    }
#pragma unroll
    for (int j = 0; j < RPT; j++) {
        const int t = t0 + g + G * j;
        if (t < T) O[((int64_t)b * T + t) * ldo + (int64_t)h * HD + d] = (int64_t)((uint64_t)acc_hi[j] + acc_lo[j]);
    }
}

template <int HD>
__global__ __launch_bounds__(PT) void k_softmax_pv(const int64_t* __restrict__ S, const int64_t* __restrict__ V,
                                                   int64_t ldv, int64_t* __restrict__ O, int64_t ldo, int T, int nh,
                                                   int nkv, const int* __restrict__ skip, int* flag) {
    constexpr int hd = HD;
    if (*skip) return;
    extern __shared__ uint8_t sm[];
    const int Tp = (T + 3) & ~3;                                   // P rows padded to 4 keys (16 B)
    uint32_t* P = (uint32_t*)sm;                                   // [PR][Tp], p in [0, 2^30]
    uint32_t* Vlo4 = P + (size_t)PR * Tp;                          // [VT][hd], 4 * (v mod 2^30)
    int32_t* Vhi = (int32_t*)(Vlo4 + (size_t)VT * hd);             // [VT][hd], v >> 30
    __shared__ int s_bad;
    const int h = blockIdx.y, b = blockIdx.z, t0 = blockIdx.x * PR;
    const int kvh = h / (nh / nkv);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) s_bad = 0;
    __syncthreads();

    // ---- softmax rows (FixedSoftmax), two rows per warp
    for (int r = warp; r < PR; r += PT / 32) {
        const int t = t0 + r;
        uint32_t* prow = P + (size_t)r * Tp;
        for (int s = T + lane; s < Tp; s += 32) prow[s] = 0;
        if (t >= T) {
            for (int s = lane; s < T; s += 32) prow[s] = 0;
            continue;
        }
        const int64_t* srow = S + (((int64_t)b * nh + h) * T + t) * T;
        int64_t mx = INT64_MIN;
        for (int s = lane; s < T; s += 32) mx = max(mx, srow[s]);
        mx = warp_max_i64(mx);
        uint64_t sum = 0;
        bool bad = false;
        for (int s = lane; s < T; s += 32) {
            int64_t e = fixed_exp30(wsub(srow[s], mx));
            bad |= e < 0 || e > (1LL << 30);
            prow[s] = (uint32_t)e;
            sum += (uint64_t)e;
        }
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, (unsigned long long)sum, o);
        bad = __any_sync(0xffffffffu, bad);
        if (bad) {
            if (lane == 0) s_bad = 1;
            continue;
        }
        __syncwarp();
        if (sum == 0) {  // uniform = one / len
            for (int s = lane; s < T; s += 32) prow[s] = (uint32_t)((1LL << 30) / T);
        } else {
            const uint64_t inv = ~0ULL / sum;
            for (int s = lane; s < T; s += 32) prow[s] = (uint32_t)udiv_inv((uint64_t)prow[s] << 30, sum, inv);
        }
    }
    __syncthreads();
    if (s_bad) {
        if (threadIdx.x == 0) atomicOr(flag, 1);
        return;
    }
    // ---- PV. Thread (g, d): d = tid % hd, rows g, g+G, ... (G = PT/hd row groups). Each key's
    // (v_hi, 4*v_lo) is read once per thread and used for all its rows; p comes four keys at a time.
    const int64_t* vb = V + (int64_t)b * T * ldv + (int64_t)kvh * hd;
    pv_rows<PR * HD / PT, HD>(P, Tp, vb, ldv, Vlo4, Vhi, T, t0, O, ldo, b, h, &s_bad);
    __syncthreads();
    if (s_bad && threadIdx.x == 0) atomicOr(flag, 1);
}

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

template <int HD>
void launch_pv(dim3 grid, size_t smem, const int64_t* scores, const int64_t* v, int64_t ldv, int64_t* out, int64_t ldo,
               int T, int nh, int nkv, int* flag, cudaStream_t st) {
    static size_t configured = 0;
    if (smem > 32 * 1024 && smem > configured) {  // opt in well before 48 KB (static smem adds to it)
        cudaFuncSetAttribute(k_softmax_pv<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        configured = smem;
    }
    k_softmax_pv<HD><<<grid, PT, smem, st>>>(scores, v, ldv, out, ldo, T, nh, nkv, flag, flag);
}
}  // namespace

size_t attention_tc_workspace(int B, int T, int nh, int nkv, int hd) {
    const int64_t kpad = round_up(hd, tc::BK);
    const int64_t qbytes = (int64_t)B * nh * tc::LA * round_up(T, tc::BM) * kpad;
    const int64_t kbytes = (int64_t)B * nkv * tc::LA * round_up(T, tc::SBN) * kpad;
    const int64_t sbytes = (int64_t)B * nh * T * T * 8;
    return (size_t)(256 + round_up(qbytes, 256) + round_up(kbytes, 256) + sbytes);
}

size_t softmax_pv_smem(int T, int hd) { return (size_t)PR * ((T + 3) & ~3) * 4 + (size_t)VT * hd * 8; }

bool attention_tc_supported(int T, int nh, int nkv, int hd) {
    const bool hd_ok = hd == 16 || hd == 32 || hd == 64 || hd == 128 || hd == 256;
    return hd_ok && nkv > 0 && nh % nkv == 0 && softmax_pv_smem(T, hd) <= 200 * 1024;
}

int attention_tc(const int64_t* q, int64_t ldq, const int64_t* k, int64_t ldk, const int64_t* v, int64_t ldv,
                 int64_t* out, int64_t ldo, int B, int T, int nh, int nkv, int hd, int score_shift, int64_t sqrt_hd,
                 int mode, int window, void* ws, int* err, cudaStream_t st) {
    const int64_t kpad = round_up(hd, tc::BK);
    const int64_t tq = round_up(T, tc::BM), tk = round_up(T, tc::SBN);
    uint8_t* base = (uint8_t*)ws;
    int* flag = (int*)base;
    int8_t* qp = (int8_t*)(base + 256);
    const int64_t qbytes = round_up((int64_t)B * nh * tc::LA * tq * kpad, 256);
    int8_t* kp = qp + qbytes;
    const int64_t kbytes = round_up((int64_t)B * nkv * tc::LA * tk * kpad, 256);
    int64_t* scores = (int64_t*)(kp + kbytes);
    alignas(64) unsigned char mq[128], mk[128];
    if (!tc::encode_planes(mq, qp, kpad, tq, tc::LA, tc::BM, (int64_t)B * nh) ||
        !tc::encode_planes(mk, kp, kpad, tk, tc::LA, tc::SBN, (int64_t)B * nkv))
        return -1;
    cudaMemsetAsync(flag, 0, sizeof(int), st);
    tc::split_heads(q, ldq, B, T, nh, hd, tq, kpad, qp, flag, st);
    tc::split_heads(k, ldk, B, T, nkv, hd, tk, kpad, kp, flag, st);
    tc::launch_scores(mq, mk, B, T, nh, nkv, tk, kpad, score_shift, sqrt_hd, mode, window, scores, flag, err, st);
    const size_t smem = softmax_pv_smem(T, hd);
    dim3 grid((unsigned)((T + PR - 1) / PR), (unsigned)nh, (unsigned)B);
    switch (hd) {
        case 16: launch_pv<16>(grid, smem, scores, v, ldv, out, ldo, T, nh, nkv, flag, st); break;
        case 32: launch_pv<32>(grid, smem, scores, v, ldv, out, ldo, T, nh, nkv, flag, st); break;
        case 64: launch_pv<64>(grid, smem, scores, v, ldv, out, ldo, T, nh, nkv, flag, st); break;
        case 128: launch_pv<128>(grid, smem, scores, v, ldv, out, ldo, T, nh, nkv, flag, st); break;
        default: launch_pv<256>(grid, smem, scores, v, ldv, out, ldo, T, nh, nkv, flag, st); break;
    }
    // the exact kernel redoes the whole call when anything fell outside the fast ranges
    attention(q, ldq, k, ldk, v, ldv, out, ldo, B, T, nh, nkv, hd, score_shift, sqrt_hd, mode, window, st, flag);
    return 6;
}

}  // namespace slx
