// k_gemv.cu -- exact decode-shaped GEMV (M <= 8 rows) straight from packed Q4_0 / Q8_0 blocks.
//
// IntegerMatMul.MatMul with the encoder's composite weights (Math/IntegerMatMul.cs:37-76,
// IntegerTransformerSource.Q): w = (long)(d * q * 2^s). For a finite f16 scale d and s >= 24 the
// product d*q*2^s is an integer, so w = D * q with D = (long)(d * 2^s), and a block's contribution is
//     sum_{k in block} a_k * w_k = D * sum_k a_k q_k.
// The inner sum runs on dp4a over the 5 balanced base-256 digits of the activations
// (a = sum_i a_i 256^i, |a_i q| <= 2^14, 32 terms per block: exact int32), combined into an
// int64 per block and multiplied by D into the Int128 accumulator. A non-finite scale makes every
// composite of its block long.MinValue, handled as D = long.MinValue with q = 1 for each element.
// Weights are read once from HBM with 16-byte copies into shared memory (each warp streams NC
// output columns' contiguous blocks); the activation digits (a few KB) stay in L1/L2 and each
// block's digits serve all NC columns.
// If any activation needs a sixth digit, the prep kernel raises the overflow word and every warp
// takes the Int128 multiply-accumulate path over the composites instead.
#include "slx_device.cuh"
#include "slx_kernels.h"

namespace slx {
namespace {

constexpr int GV_THREADS = 256;
constexpr int ND = 5;  // activation digits

// Activation digits for the GEMV: dig[m][i][k] (int8) in the element order a block's 32-bit
// words present: for Q4_0 word j of a block carries elements (8j, 8j+2, 8j+4, 8j+6) in its low
// nibbles and (8j+1, ..., 8j+7) in its high nibbles; Q8_0 words carry elements in order.
// Also bsum[m][i][blk] = sum of digit i over the block (for the Q4_0 offset of 8).
__global__ void k_gemv_prep(const int64_t* __restrict__ A, int64_t lda, int M, int K, int q4, int8_t* __restrict__ dig,
                            int* __restrict__ bsum, int* overflow) {
    const int nb = K / 32;
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;  // over M * nb blocks
    if (idx >= M * nb) return;
    const int m = idx / nb, blk = idx % nb;
    int8_t d[ND][32];
    int sum[ND] = {0, 0, 0, 0, 0};
    bool bad = false;
    for (int e = 0; e < 32; e++) {
        int64_t x = A[(int64_t)m * lda + (int64_t)blk * 32 + e];
        // position of element e inside the block's byte stream
        int pos;
        if (q4) {
            const int j = e >> 3, r = e & 7;          // word j, r-th element of the word
            pos = j * 8 + ((r & 1) ? 4 : 0) + (r >> 1);  // even elements first (low nibbles), then odd
        } else {
            pos = e;
        }
#pragma unroll
        for (int i = 0; i < ND; i++) {
            int dd = (int)(((uint64_t)x + 128u) & 255u) - 128;
            x = (x - dd) >> 8;
            d[i][pos] = (int8_t)dd;
            sum[i] += dd;
        }
        bad |= x != 0;
    }
    if (bad) atomicOr(overflow, 1);
    for (int i = 0; i < ND; i++) {
        int8_t* dst = dig + ((int64_t)m * ND + i) * K + (int64_t)blk * 32;
        for (int e = 0; e < 32; e++) dst[e] = d[i][e];
        bsum[((int64_t)m * ND + i) * nb + blk] = sum[i];
    }
}

SLX_DEV int dp4a_su(int a_signed, unsigned b_unsigned, int c) {
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_signed), "r"(b_unsigned), "r"(c));
    return d;
}

// One block's 8 words of 4 bytes: Q4_0 nibbles unpacked to (low nibbles, high nibbles) of 4 words,
// Q8_0 signed bytes as they are. Returns the block's scale bits.
template <bool Q4>
SLX_DEV uint16_t load_block(const uint8_t* __restrict__ blk, uint32_t (&w)[8]) {
    const uint16_t* h = (const uint16_t*)blk;
    const uint16_t scale = h[0];
    if (Q4) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint32_t x = (uint32_t)h[1 + 2 * j] | ((uint32_t)h[2 + 2 * j] << 16);
            w[2 * j] = x & 0x0F0F0F0Fu;             // elements 8j, 8j+2, 8j+4, 8j+6 (nibble values 0..15)
            w[2 * j + 1] = (x >> 4) & 0x0F0F0F0Fu;  // elements 8j+1, ..., 8j+7
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; j++) w[j] = (uint32_t)h[1 + 2 * j] | ((uint32_t)h[2 + 2 * j] << 16);
    }
    return scale;
}

// Warp = NC output columns. The warp streams its columns' packed blocks through shared memory in
// chunks of 64 blocks with 16-byte cp.async copies (double buffered, so the next chunk is in flight
// while this one is decoded); lane l decodes blocks l and l+32 of each chunk. Row starts and chunk
// starts are 16-byte aligned when K is a multiple of 256 (checked by the launcher).
constexpr int GV_CHUNK = 64;  // blocks per chunk

SLX_DEV void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)), "l"(gmem)
                 : "memory");
}
SLX_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
SLX_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <bool Q4, int MM, int NC>
__global__ __launch_bounds__(GV_THREADS) void k_gemv(const uint8_t* __restrict__ W, int N, int K, const int8_t* __restrict__ dig,
                                                     const int* __restrict__ bsum, int64_t* __restrict__ C, int64_t ldc,
                                                     int shift, const int* __restrict__ skip,
                                                     const int64_t* __restrict__ A, int64_t lda, double scale) {
    constexpr int BB = Q4 ? 18 : 34;
    constexpr int CHB = GV_CHUNK * BB;       // bytes per column chunk (multiple of 16)
    if (*skip) {  // an activation needs a sixth digit: Int128 multiply-accumulate of the composites
        const int warp_ = threadIdx.x >> 5, lane_ = threadIdx.x & 31;
        const int nb0 = (blockIdx.x * (GV_THREADS / 32) + warp_) * NC;
        const int64_t nblk = K / 32;
        for (int c = 0; c < NC && nb0 + c < N; c++) {
            for (int m = 0; m < MM; m++) {
                u128 a128 = 0;
                for (int k = lane_; k < K; k += 32) {
                    const int64_t e = (int64_t)(nb0 + c) * K + k;
                    const int64_t wq = composite(dequant_elem(Q4 ? DT_Q4_0 : DT_Q8_0, W, e, nblk * N), 0, scale);
                    a128 += (u128)((i128)A[(int64_t)m * lda + k] * wq);
                }
                a128 = warp_sum_u128(a128);
                if (lane_ == 0) C[(int64_t)m * ldc + nb0 + c] = shift > 0 ? lo64(sar128((i128)a128, shift)) : lo64((i128)a128);
            }
        }
        return;
    }
    constexpr int VEC = CHB / 16;            // 16-byte copies per column chunk
    extern __shared__ __align__(16) uint8_t gv_smem[];
    const int nb = K / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = (blockIdx.x * (GV_THREADS / 32) + warp) * NC;
    if (n0 >= N) return;
    uint8_t* buf = gv_smem + (size_t)warp * 2 * NC * CHB;  // [2][NC][CHB]
    const int nchunks = (nb + GV_CHUNK - 1) / GV_CHUNK;

    auto issue = [&](int ch) {
        uint8_t* dst = buf + (ch & 1) * NC * CHB;
        const int blocks = min(GV_CHUNK, nb - ch * GV_CHUNK);
        const int vecs = (blocks * BB + 15) / 16;
#pragma unroll
        for (int c = 0; c < NC; c++) {
            const int n = min(n0 + c, N - 1);
            const uint8_t* src = W + ((int64_t)n * nb + (int64_t)ch * GV_CHUNK) * BB;
            for (int v = lane; v < vecs; v += 32) cp_async16(dst + c * CHB + v * 16, src + v * 16);
        }
        cp_async_commit();
    };

    u128 acc[MM][NC];
#pragma unroll
    for (int m = 0; m < MM; m++)
#pragma unroll
        for (int c = 0; c < NC; c++) acc[m][c] = 0;
    issue(0);
    for (int ch = 0; ch < nchunks; ch++) {
        if (ch + 1 < nchunks) {
            issue(ch + 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncwarp();
        const uint8_t* cur = buf + (ch & 1) * NC * CHB;
        const int blocks = min(GV_CHUNK, nb - ch * GV_CHUNK);
#pragma unroll
        for (int half = 0; half < 2; half++) {
            const int lb = lane + 32 * half;
            if (lb >= blocks) break;
            const int blk = ch * GV_CHUNK + lb;
            uint32_t w[NC][8];
            int64_t D[NC];
            bool fin[NC];
#pragma unroll
            for (int c = 0; c < NC; c++) {
                const uint16_t sbits = load_block<Q4>(cur + c * CHB + lb * BB, w[c]);
                const float d = h2f(sbits);
                fin[c] = isfinite(d);
                D[c] = fin[c] ? (int64_t)((double)d * scale) : INT64_MIN;
            }
#pragma unroll
            for (int m = 0; m < MM; m++) {
                int64_t S[NC];
#pragma unroll
                for (int c = 0; c < NC; c++) S[c] = 0;
#pragma unroll
                for (int i = ND - 1; i >= 0; i--) {
                    const int8_t* dg = dig + ((int64_t)m * ND + i) * K + (int64_t)blk * 32;
                    const int4 a0 = __ldg((const int4*)dg), a1 = __ldg((const int4*)(dg + 16));
                    const int av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                    const int bs = __ldg(bsum + ((int64_t)m * ND + i) * nb + blk);
#pragma unroll
                    for (int c = 0; c < NC; c++) {
                        int p = 0;
#pragma unroll
                        for (int j = 0; j < 8; j++) p = Q4 ? dp4a_su(av[j], w[c][j], p) : __dp4a(av[j], (int)w[c][j], p);
                        if (Q4) p -= 8 * bs;
                        if (!fin[c]) p = bs;  // every composite of the block is long.MinValue
                        S[c] = S[c] * 256 + p;  // digits combined high to low: |S| < 2^59
                    }
                }
#pragma unroll
                for (int c = 0; c < NC; c++) acc[m][c] += (u128)((i128)S[c] * D[c]);
            }
        }
        __syncwarp();  // this buffer is refilled two chunks later
    }
#pragma unroll
    for (int m = 0; m < MM; m++)
#pragma unroll
        for (int c = 0; c < NC; c++) {
            const u128 v = warp_sum_u128(acc[m][c]);
            if (lane == 0 && n0 + c < N)
                C[(int64_t)m * ldc + n0 + c] = shift > 0 ? lo64(sar128((i128)v, shift)) : lo64((i128)v);
        }
}

template <bool Q4, int MM, int NC>
void launch_one(const uint8_t* w, int N, int K, const int8_t* dig, const int* bsum, int64_t* c, int64_t ldc, int shift,
                const int* skip, const int64_t* a, int64_t lda, double scale, cudaStream_t st) {
    const int cols_per_block = (GV_THREADS / 32) * NC;
    dim3 grid((unsigned)((N + cols_per_block - 1) / cols_per_block));
    const size_t smem = (size_t)(GV_THREADS / 32) * 2 * NC * GV_CHUNK * (Q4 ? 18 : 34);
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(k_gemv<Q4, MM, NC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        configured = true;
    }
    k_gemv<Q4, MM, NC><<<grid, GV_THREADS, smem, st>>>(w, N, K, dig, bsum, c, ldc, shift, skip, a, lda, scale);
}

template <bool Q4>
void launch_gemv_m(int M, const uint8_t* w, int N, int K, const int8_t* dig, const int* bsum, int64_t* c, int64_t ldc,
                   int shift, const int* skip, const int64_t* a, int64_t lda, double scale, cudaStream_t st) {
    switch (M) {
        case 1: launch_one<Q4, 1, 4>(w, N, K, dig, bsum, c, ldc, shift, skip, a, lda, scale, st); break;
        case 2: launch_one<Q4, 2, 4>(w, N, K, dig, bsum, c, ldc, shift, skip, a, lda, scale, st); break;
        case 3: launch_one<Q4, 3, 2>(w, N, K, dig, bsum, c, ldc, shift, skip, a, lda, scale, st); break;
        case 4: launch_one<Q4, 4, 2>(w, N, K, dig, bsum, c, ldc, shift, skip, a, lda, scale, st); break;
        case 5: launch_one<Q4, 5, 1>(w, N, K, dig, bsum, c, ldc, shift, skip, a, lda, scale, st); break;
        case 6: launch_one<Q4, 6, 1>(w, N, K, dig, bsum, c, ldc, shift, skip, a, lda, scale, st); break;
        case 7: launch_one<Q4, 7, 1>(w, N, K, dig, bsum, c, ldc, shift, skip, a, lda, scale, st); break;
        default: launch_one<Q4, 8, 1>(w, N, K, dig, bsum, c, ldc, shift, skip, a, lda, scale, st); break;
    }
}

}  // namespace

bool gemv_supported(const WDesc& w, int M) {
    // d * 2^s is an integer for every f16 d only when s >= 24 (the smallest subnormal is 2^-24)
    return M >= 1 && M <= 8 && w.mode == 0 && (w.dtype == DT_Q4_0 || w.dtype == DT_Q8_0) && w.K % 256 == 0 &&
           w.scale >= 16777216.0 &&
           w.nblocks * 32 >= w.N * w.K && ((uintptr_t)w.data & 15) == 0;
}

size_t gemv_workspace(int M, int K) { return 256 + (size_t)M * ND * K + (size_t)M * ND * (K / 32) * 4 + 256; }

namespace {
struct GemvWs {
    int* flag;
    int8_t* dig;
    int* bsum;
};
GemvWs gemv_ws(void* ws, int M, int K) {
    GemvWs g;
    g.flag = (int*)ws;
    g.dig = (int8_t*)ws + 256;
    g.bsum = (int*)(g.dig + (((size_t)M * ND * K + 255) & ~(size_t)255));
    return g;
}
}  // namespace

int gemv_prep(const int64_t* a, int64_t lda, int M, const WDesc& w, void* ws, cudaStream_t st) {
    const int K = (int)w.K, nb = K / 32;
    GemvWs g = gemv_ws(ws, M, K);
    cudaMemsetAsync(g.flag, 0, sizeof(int), st);
    k_gemv_prep<<<(M * nb + 127) / 128, 128, 0, st>>>(a, lda, M, K, w.dtype == DT_Q4_0, g.dig, g.bsum, g.flag);
    return 1;
}

int gemv_main(const int64_t* a, int64_t lda, int M, const WDesc& w, int64_t* c, int64_t ldc, int shift, void* ws,
              cudaStream_t st) {
    const int K = (int)w.K, N = (int)w.N;
    GemvWs g = gemv_ws(ws, M, K);
    if (w.dtype == DT_Q4_0)
        launch_gemv_m<true>(M, w.data, N, K, g.dig, g.bsum, c, ldc, shift, g.flag, a, lda, w.scale, st);
    else
        launch_gemv_m<false>(M, w.data, N, K, g.dig, g.bsum, c, ldc, shift, g.flag, a, lda, w.scale, st);
    return 1;
}

int gemv_exact(const int64_t* a, int64_t lda, int M, const WDesc& w, int64_t* c, int64_t ldc, int shift, void* ws,
               cudaStream_t st) {
    return gemv_prep(a, lda, M, w, ws, st) + gemv_main(a, lda, M, w, c, ldc, shift, ws, st);
}

}  // namespace slx
