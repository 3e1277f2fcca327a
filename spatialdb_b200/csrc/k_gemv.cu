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
// If any activation needs a sixth digit, the prep kernel stores its call's tag in the overflow word
// and every warp takes the Int128 multiply-accumulate path over the composites instead.
#include "slx_device.cuh"
#include "slx_gemm.h"
#include "slx_kernels.h"

namespace slx {
namespace {

constexpr int GV_THREADS = 256;
constexpr int ND = 5;  // activation digits
constexpr int FLAG_WORD = 16;  // int index of the GEMV overflow word in the workspace

// Activation digits for the GEMV, dig[m][blk][i][32] (int8, 160 contiguous bytes per row and
// block), in the element order a block's 32-bit words present: for Q4_0 word j of a block carries
// elements (8j, 8j+2, 8j+4, 8j+6) in its low nibbles and (8j+1, ..., 8j+7) in its high nibbles;
// Q8_0 words carry elements in order. asum[m][blk] = sum of the block's activations (wrapping),
// used for the Q4_0 offset of 8 and for non-finite scales. Four threads per (row, block), each
// splitting 8 consecutive activations. An activation that needs a sixth digit stores `tag` in the
// overflow word.
__global__ void k_gemv_prep(const int64_t* __restrict__ A, int64_t lda, int M, int K, int q4, int8_t* __restrict__ dig,
                            int64_t* __restrict__ asum, int* overflow, int tag) {
    const int nb = K / 32;
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    const int pair = t >> 2, j = t & 3;  // pair = m * nb + blk; blocks of 4 threads stay inside one warp
    const bool live = pair < M * nb;
    const int m = live ? pair / nb : 0, blk = live ? pair % nb : 0;
    int64_t x[8];
    int64_t sum = 0;
#pragma unroll
    for (int e = 0; e < 8; e++) {
        x[e] = live ? A[(int64_t)m * lda + (int64_t)blk * 32 + 8 * j + e] : 0;
        sum = wadd(sum, x[e]);
    }
    uint32_t lo[ND], hi[ND];
#pragma unroll
    for (int i = 0; i < ND; i++) lo[i] = hi[i] = 0;
    bool bad = false;
#pragma unroll
    for (int e = 0; e < 8; e++) {
        int64_t v = x[e];
        // Q4_0: even elements go to the low-nibble word, odd ones to the high-nibble word;
        // Q8_0: elements 0..3 to the first word, 4..7 to the second.
        const int word = q4 ? (e & 1) : (e >> 2);
        const int byte = q4 ? (e >> 1) : (e & 3);
#pragma unroll
        for (int i = 0; i < ND; i++) {
            const int d = (int)(((uint64_t)v + 128u) & 255u) - 128;
            v = (v - d) >> 8;
            const uint32_t b = (uint32_t)(uint8_t)(int8_t)d << (8 * byte);
            if (word) hi[i] |= b; else lo[i] |= b;
        }
        bad |= v != 0;
    }
    sum = wadd(sum, (int64_t)__shfl_xor_sync(0xffffffffu, (long long)sum, 1));
    sum = wadd(sum, (int64_t)__shfl_xor_sync(0xffffffffu, (long long)sum, 2));
    if (!live) return;
    if (bad) atomicExch(overflow, tag);
    int8_t* dst = dig + (int64_t)pair * (ND * 32) + 8 * j;
#pragma unroll
    for (int i = 0; i < ND; i++) *(uint2*)(dst + i * 32) = make_uint2(lo[i], hi[i]);
    if (j == 0) asum[pair] = sum;
}

SLX_DEV int dp4a_su(int a_signed, unsigned b_unsigned, int c) {
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_signed), "r"(b_unsigned), "r"(c));
    return d;
}

// One block's 8 words of 4 bytes from shared memory: Q4_0 nibbles unpacked to (low nibbles, high
// nibbles) of 4 words, Q8_0 signed bytes as they are. Returns the block's scale bits. Blocks are 18 or
// 34 bytes, so a block starts on a 4-byte boundary or 2 bytes past one: the words are read aligned
// and funnel-shifted by 16 bits (or taken as they are, a clamped shift of 32).
template <bool Q4>
SLX_DEV uint16_t load_block(const uint8_t* __restrict__ blk, uint32_t (&w)[8]) {
    constexpr int NW = Q4 ? 5 : 9;
    const uint32_t* p = (const uint32_t*)((uintptr_t)blk & ~(uintptr_t)3);
    const uint32_t s = ((uintptr_t)blk & 2) ? 32u : 16u;
    uint32_t r[NW];
#pragma unroll
    for (int i = 0; i < NW; i++) r[i] = p[i];
    const uint16_t scale = (uint16_t)(r[0] >> (s - 16));
    if (Q4) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint32_t x = __funnelshift_rc(r[j], r[j + 1], s);
            w[2 * j] = x & 0x0F0F0F0Fu;             // elements 8j, 8j+2, 8j+4, 8j+6 (nibble values 0..15)
            w[2 * j + 1] = (x >> 4) & 0x0F0F0F0Fu;  // elements 8j+1, ..., 8j+7
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; j++) w[j] = __funnelshift_rc(r[j], r[j + 1], s);
    }
    return scale;
}

// acc += (Int128)s * d
SLX_DEV void mac128(u128& acc, int64_t s, int64_t d) {
    const uint64_t lo = (uint64_t)s * (uint64_t)d;
    const int64_t hi = __mul64hi(s, d);
    acc += ((u128)(uint64_t)hi << 64) | lo;
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
                                                     const int64_t* __restrict__ asum, int64_t* __restrict__ C, int64_t ldc,
                                                     int shift, const int* __restrict__ skip, int tag,
                                                     const int64_t* __restrict__ A, int64_t lda, double scale) {
    constexpr int BB = Q4 ? 18 : 34;
    constexpr int CHB = GV_CHUNK * BB;       // bytes per column chunk (multiple of 16)
    if (*skip == tag) {  // an activation needs a sixth digit: Int128 multiply-accumulate of the composites
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
                const int8_t* dg = dig + ((int64_t)m * nb + blk) * (ND * 32);
                int4 dv[ND][2];
#pragma unroll
                for (int i = 0; i < ND; i++) {
                    dv[i][0] = __ldg((const int4*)(dg + 32 * i));
                    dv[i][1] = __ldg((const int4*)(dg + 32 * i + 16));
                }
                const int64_t as = __ldg(asum + (int64_t)m * nb + blk);
#pragma unroll
                for (int c = 0; c < NC; c++) {
                    int P[ND];
#pragma unroll
                    for (int i = 0; i < ND; i++) {
                        const int av[8] = {dv[i][0].x, dv[i][0].y, dv[i][0].z, dv[i][0].w,
                                           dv[i][1].x, dv[i][1].y, dv[i][1].z, dv[i][1].w};
                        int p = 0;
#pragma unroll
                        for (int jj = 0; jj < 8; jj++)
                            p = Q4 ? dp4a_su(av[jj], w[c][jj], p) : __dp4a(av[jj], (int)w[c][jj], p);
                        P[i] = p;
                    }
                    // sum_i 256^i P_i: |P_i| < 2^17, so the two low pairs combine in 32 bits
                    const int t01 = P[1] * 256 + P[0], t23 = P[3] * 256 + P[2];
                    int64_t S = (int64_t)t01 + (int64_t)t23 * 65536 + ((int64_t)P[4] << 32);
                    if (Q4) S -= 8 * as;    // nibble q - 8
                    if (!fin[c]) S = as;    // every composite of the block is long.MinValue
                    mac128(acc[m][c], S, D[c]);
                }
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
void launch_one(const uint8_t* w, int N, int K, const int8_t* dig, const int64_t* asum, int64_t* c, int64_t ldc, int shift,
                const int* skip, int tag, const int64_t* a, int64_t lda, double scale, cudaStream_t st) {
    const int cols_per_block = (GV_THREADS / 32) * NC;
    dim3 grid((unsigned)((N + cols_per_block - 1) / cols_per_block));
    const size_t smem = (size_t)(GV_THREADS / 32) * 2 * NC * GV_CHUNK * (Q4 ? 18 : 34);
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(k_gemv<Q4, MM, NC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        configured = true;
    }
    k_gemv<Q4, MM, NC><<<grid, GV_THREADS, smem, st>>>(w, N, K, dig, asum, c, ldc, shift, skip, tag, a, lda, scale);
}

template <bool Q4>
void launch_gemv_m(int M, const uint8_t* w, int N, int K, const int8_t* dig, const int64_t* asum, int64_t* c,
                   int64_t ldc, int shift, const int* skip, int tag, const int64_t* a, int64_t lda, double scale,
                   cudaStream_t st) {
#define SLX_GV(MM, NC) launch_one<Q4, MM, NC>(w, N, K, dig, asum, c, ldc, shift, skip, tag, a, lda, scale, st)
    switch (M) {
        case 1: SLX_GV(1, 4); break;
        case 2: SLX_GV(2, 4); break;
        case 3: SLX_GV(3, 2); break;
        case 4: SLX_GV(4, 2); break;
        case 5: SLX_GV(5, 1); break;
        case 6: SLX_GV(6, 1); break;
        case 7: SLX_GV(7, 1); break;
        default: SLX_GV(8, 1); break;
    }
#undef SLX_GV
}

// Workspace: [0, 256) flags (the GEMV overflow word at int index FLAG_WORD), then the digits
// (M * K * 5 bytes), then the per-block activation sums (M * K / 32 int64).
struct GemvWs {
    int* flag;
    int8_t* dig;
    int64_t* asum;
};
GemvWs gemv_ws(void* ws, int M, int K) {
    GemvWs g;
    g.flag = (int*)ws + FLAG_WORD;
    g.dig = (int8_t*)ws + 256;
    g.asum = (int64_t*)(g.dig + (((size_t)M * ND * K + 255) & ~(size_t)255));
    return g;
}
size_t gemv_workspace(int M, int K) { return 256 + (((size_t)M * ND * K + 255) & ~(size_t)255) + (size_t)M * (K / 32) * 8; }

}  // namespace

bool gemv_supported(const WDesc& w, int M) {
    // d * 2^s is an integer for every f16 d only when s >= 24 (the smallest subnormal is 2^-24)
    return M >= 1 && M <= 8 && w.mode == 0 && (w.dtype == DT_Q4_0 || w.dtype == DT_Q8_0) && w.K % 256 == 0 &&
           w.scale >= 16777216.0 &&
           w.nblocks * 32 >= w.N * w.K && ((uintptr_t)w.data & 15) == 0;
}

bool gemv_reserve(GemmWorkspace& ws, int M, int K, cudaStream_t st) {
    const size_t need = gemv_workspace(M, K);
    if (need <= ws.bytes) return true;
    if (ws.p) cudaFree(ws.p);
    ws.p = nullptr;
    ws.bytes = 0;
    ws.tag = 0;
    if (cudaMalloc(&ws.p, need) != cudaSuccess) return false;
    ws.bytes = need;
    cudaMemsetAsync(ws.p, 0, 256, st);  // overflow words start below every tag
    return true;
}

int gemv_prep(const int64_t* a, int64_t lda, int M, const WDesc& w, GemmWorkspace& ws, cudaStream_t st) {
    const int K = (int)w.K, nb = K / 32;
    GemvWs g = gemv_ws(ws.p, M, K);
    ws.tag = ws.tag >= 0x3fffffff ? 1 : ws.tag + 1;  // never 0, the cleared value
    const int threads = M * nb * 4;
    k_gemv_prep<<<(threads + 127) / 128, 128, 0, st>>>(a, lda, M, K, w.dtype == DT_Q4_0, g.dig, g.asum, g.flag,
                                                       (int)ws.tag);
    return 1;
}

int gemv_main(const int64_t* a, int64_t lda, int M, const WDesc& w, int64_t* c, int64_t ldc, int shift,
              const GemmWorkspace& ws, cudaStream_t st) {
    const int K = (int)w.K, N = (int)w.N;
    GemvWs g = gemv_ws(ws.p, M, K);
    if (w.dtype == DT_Q4_0)
        launch_gemv_m<true>(M, w.data, N, K, g.dig, g.asum, c, ldc, shift, g.flag, (int)ws.tag, a, lda, w.scale, st);
    else
        launch_gemv_m<false>(M, w.data, N, K, g.dig, g.asum, c, ldc, shift, g.flag, (int)ws.tag, a, lda, w.scale, st);
    return 1;
}

int gemv_exact(const int64_t* a, int64_t lda, int M, const WDesc& w, int64_t* c, int64_t ldc, int shift,
               GemmWorkspace& ws, cudaStream_t st) {
    return gemv_prep(a, lda, M, w, ws, st) + gemv_main(a, lda, M, w, c, ldc, shift, ws, st);
}

}  // namespace slx
