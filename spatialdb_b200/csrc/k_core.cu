// k_core.cu -- exact integer kernels of the SparseLattice forward path on CUDA cores.
//
// Every kernel reproduces the reference's integer results bit for bit (C# unchecked long /
// Int128 arithmetic, truncating division, flooring shifts). The tensor-core GEMM in k_gemm_tc.cu
// replaces gemm_exact on the hot path; this file keeps the exact general path that any
// activation range falls back to.
#include <algorithm>
#include <cstdio>

#include "slx_attr.h"
#include "slx_device.cuh"
#include "slx_exact.cuh"
#include "slx_kernels.h"

namespace slx {

// ------------------------------------------------------------------------------------------
// GEMM: c = (a . w^T) >> shift (+ r)    IntegerMatMul.MatMul + DotInt128 (IntegerMatMul.cs:37-76,
// 209-229) with the weight's Q30 composite formed in-kernel from the packed GGUF blocks.
// 64x64 output tile, K in steps of one 32-element quant block, 4x4 Int128 accumulators per thread.
// ------------------------------------------------------------------------------------------
namespace {
__global__ __launch_bounds__(XTH) void k_gemm_exact(const int64_t* __restrict__ A, int64_t lda, int M, int K, WDesc W,
                                                    int64_t* __restrict__ C, int64_t ldc, int shift,
                                                    const int64_t* __restrict__ R, int64_t ldr,
                                                    const int* __restrict__ only_if) {
    if (only_if && *only_if == 0) return;
    __shared__ int64_t As[XBK][XBM + 1];
    __shared__ int64_t Ws[XBK][XBN + 1];
    exact_gemm_tiles(A, lda, M, K, W, C, ldc, shift, R, ldr, As, Ws, blockIdx.x, gridDim.x);
}

__global__ void k_weight_q30(WDesc W, int64_t n, int64_t* out) {
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i < n) out[i] = composite(dequant_elem(W.dtype, W.data, i, W.nblocks), W.mode, W.scale);
}
}  // namespace

int gemm_exact(const int64_t* a, int64_t lda, int M, int K, const WDesc& w, int64_t* c, int64_t ldc, int shift,
                const int64_t* r, int64_t ldr, cudaStream_t st, const int* only_if) {
    if (M <= 0 || w.N <= 0) return 0;
    const int64_t ntiles = ((w.N + XBN - 1) / XBN) * (int64_t)((M + XBM - 1) / XBM);
    // Gated behind a faster path it usually does nothing, so a small grid walks the tiles.
    const int64_t grid = only_if ? std::min<int64_t>(ntiles, 2 * 148) : ntiles;
    k_gemm_exact<<<(unsigned)grid, XTH, 0, st>>>(a, lda, M, K, w, c, ldc, shift, r, ldr, only_if);
    return 1;
}

int weight_to_q30(const WDesc& w, int64_t n, int64_t* out, cudaStream_t st) {
    if (n <= 0) return 0;
    k_weight_q30<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(w, n, out);
    return 1;
}

// ------------------------------------------------------------------------------------------
// GgufDequantizer formulas for every decodable dtype (GgufDequantizer.cs:7-325), one element per
// thread, float arithmetic in the reference's order without contraction.
// ------------------------------------------------------------------------------------------
namespace {
__device__ __constant__ float c_mxfp4[15] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                                             -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -10.0f};

SLX_DEV void q4k_scale(const uint8_t* raw, int j, int& sc, int& m) {  // UnpackQ4KScales (:345-357)
    if (j < 4) {
        sc = raw[j] & 63;
        m = raw[j + 4] & 63;
    } else {
        sc = (raw[j + 4] & 0x0F) | ((raw[j - 4] >> 6) << 4);
        m = (raw[j + 4] >> 4) | ((raw[j] >> 6) << 4);
    }
}

__global__ void k_dequant_f32(int dtype, const uint8_t* __restrict__ raw, int64_t n, float* __restrict__ out,
                              int* flag) {
    int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (e >= n) return;
    float v = 0.0f;
    switch (dtype) {
        case 0: v = ((const float*)raw)[e]; break;
        case 1: v = h2f(((const uint16_t*)raw)[e]); break;
        case 30: v = __uint_as_float((uint32_t)((const uint16_t*)raw)[e] << 16); break;
        case 8: case 2: v = dequant_elem(dtype, raw, e, n / 32); break;
        case 39: {  // DequantizeMXFP4 (:97-123)
            int64_t b = e >> 5;
            if (b >= n / 32) break;
            const uint8_t* blk = raw + b * 17;
            int j = (int)(e & 31);
            uint8_t byte = blk[1 + (j >> 1)];
            // The reference decodes lo then hi of each byte; an out-of-range nibble throws.
            int nib = (j & 1) ? ((byte >> 4) & 0x0F) : (byte & 0x0F);
            uint8_t e8 = blk[0];
            float shared = e8 == 0 ? 0.0f : ldexpf(1.0f, (int)e8 - 127);
            if (nib >= 15) { atomicOr(flag, KERR_RANGE); break; }
            v = __fmul_rn(c_mxfp4[nib], shared);
            break;
        }
        case 10: {  // DequantizeQ2K (:125-156)
            int64_t sb = e >> 8;
            if (sb >= n / 256) break;
            const uint8_t* s = raw + sb * 84;
            int j = (int)(e & 255);
            float d = h2f(ld_u16(s)), dmin = h2f(ld_u16(s + 2));
            uint8_t scb = s[4 + j / 16];
            int q = (s[20 + j / 4] >> ((j % 4) * 2)) & 3;
            v = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)(scb & 0x0F)), (float)q), __fmul_rn(dmin, (float)(scb >> 4)));
            break;
        }
        case 11: {  // DequantizeQ3K (:158-199)
            int64_t sb = e >> 8;
            if (sb >= n / 256) break;
            const uint8_t* s = raw + sb * 110;
            int j = (int)(e & 255), g = j / 16;
            const uint8_t* sc = s + 96;
            int low4 = (g < 8) ? (sc[g] & 0x0F) : (sc[g - 8] >> 4);
            int high2 = (sc[8 + g / 4] >> (2 * (g % 4))) & 3;
            int scale = (low4 | (high2 << 4)) - 32;
            int q = ((s[32 + j / 4] >> ((j % 4) * 2)) & 3) | (((s[j / 8] >> (j % 8)) & 1) << 2);
            float d = h2f(ld_u16(s + 108));
            v = __fmul_rn(__fmul_rn(d, (float)scale), (float)(q - 4));
            break;
        }
        case 12: case 13: {  // DequantizeQ4K (:201-232), DequantizeQ5K (:234-268)
            bool q5 = dtype == 13;
            int64_t sb = e >> 8;
            if (sb >= n / 256) break;
            const uint8_t* s = raw + sb * (q5 ? 176 : 144);
            int j = (int)(e & 255), sub = j / 32;
            int sc, m;
            q4k_scale(s + 4, sub, sc, m);
            int qb = s[(q5 ? 48 : 16) + j / 2];
            int q = (j % 2 == 0) ? (qb & 0x0F) : (qb >> 4);
            if (q5) q |= ((s[16 + j / 8] >> (j % 8)) & 1) << 4;
            float d = h2f(ld_u16(s)), dmin = h2f(ld_u16(s + 2));
            v = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)m));
            break;
        }
        case 14: {  // DequantizeQ6K (:270-303)
            int64_t sb = e >> 8;
            if (sb >= n / 256) break;
            const uint8_t* s = raw + sb * 210;
            int j = (int)(e & 255);
            int8_t sc = (int8_t)s[192 + j / 16];
            int qb = s[j / 2];
            int q = ((j % 2 == 0) ? (qb & 0x0F) : (qb >> 4)) | (((s[128 + j / 4] >> ((j % 4) * 2)) & 3) << 4);
            float d = h2f(ld_u16(s + 208));
            v = __fmul_rn(__fmul_rn(d, (float)sc), (float)(q - 32));
            break;
        }
        case 15: {  // DequantizeQ8K (:305-325)
            int64_t sb = e >> 8;
            if (sb >= n / 256) break;
            const uint8_t* s = raw + sb * 292;
            float d;
            memcpy(&d, s, 4);
            v = __fmul_rn(d, (float)(int8_t)s[4 + (e & 255)]);
            break;
        }
    }
    out[e] = v;
}
}  // namespace

int dequant_f32(int dtype, const uint8_t* raw, int64_t n, float* out, int* flag, cudaStream_t st) {
    if (n <= 0) return 0;
    k_dequant_f32<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(dtype, raw, n, out, flag);
    return 1;
}

// ------------------------------------------------------------------------------------------
// Embeddings
// ------------------------------------------------------------------------------------------
namespace {
// IntegerTransformerSource.BuildEmbeddings (IntegerTransformerSource.Forward.cs:7-26)
__global__ void k_embed_encoder(const int32_t* __restrict__ ids, int T, WDesc tok, const int64_t* __restrict__ tt,
                                int unk, int64_t* __restrict__ x, int* flag) {
    int row = blockIdx.x;
    int d = (int)tok.K;
    int id = ids[row];
    int64_t src = (int64_t)id * d;
    if (id < 0 || src + d > tok.elements) src = (int64_t)unk * d;
    bool bad = unk < 0 || src + d > tok.elements;
    if (bad && threadIdx.x == 0) atomicOr(flag, KERR_RANGE);
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
        int64_t e = bad ? 0 : composite(dequant_elem(tok.dtype, tok.data, src + j, tok.nblocks), tok.mode, tok.scale);
        x[(int64_t)row * d + j] = wadd(e, tt[j]);
    }
}

// IntegerCausalSource.BuildEmbeddings (IntegerCausalSource.Forward.cs:7-31) with a Half composite;
// IntegerGemmaSource.BuildEmbeddings (IntegerGemmaSource.Forward.cs:7-30) with a long composite.
__global__ void k_embed_scaled(const int32_t* __restrict__ ids, WDesc tok, int unk, int64_t sqrt_d,
                               int64_t* __restrict__ x, int* flag) {
    int row = blockIdx.x;
    int d = (int)tok.K;
    int id = ids[row];
    int64_t src = (int64_t)id * d;
    if (id < 0 || src + d > tok.elements) src = (int64_t)unk * d;
    bool bad = unk < 0 || src + d > tok.elements;
    if (bad && threadIdx.x == 0) atomicOr(flag, KERR_RANGE);
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
        int64_t e = bad ? 0 : composite(dequant_elem(tok.dtype, tok.data, src + j, tok.nblocks), tok.mode, tok.scale);
        x[(int64_t)row * d + j] = lo64((i128)e * sqrt_d);
    }
}
}  // namespace

int embed_encoder(const int32_t* ids, int B, int T, const WDesc& tok, const int64_t* tt, int unk, int64_t* x,
                   int* flag, cudaStream_t st) {
    if (B * T <= 0) return 0;
    k_embed_encoder<<<B * T, 256, 0, st>>>(ids, T, tok, tt, unk, x, flag);
    return 1;
}

int embed_scaled(const int32_t* ids, int B, int T, const WDesc& tok, int unk, int64_t sqrt_d, int64_t* x, int* flag,
                  cudaStream_t st) {
    if (B * T <= 0) return 0;
    k_embed_scaled<<<B * T, 256, 0, st>>>(ids, tok, unk, sqrt_d, x, flag);
    return 1;
}

// ------------------------------------------------------------------------------------------
// Norms (IntegerLayerNorm.cs)
// ------------------------------------------------------------------------------------------
namespace {
constexpr int NT = 256;

SLX_DEV u128 block_sum_u128(u128 v, u128* sh) {
    v = warp_sum_u128(v);
    int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) sh[w] = v;
    __syncthreads();
    u128 t = 0;
    if (threadIdx.x < 32) {
        t = (threadIdx.x < (blockDim.x >> 5)) ? sh[threadIdx.x] : 0;
        t = warp_sum_u128(t);
        if (threadIdx.x == 0) sh[0] = t;
    }
    __syncthreads();
    t = sh[0];
    __syncthreads();
    return t;
}

// NormalizeRow (IntegerLayerNorm.cs:21-57)
__global__ __launch_bounds__(NT) void k_layernorm(int64_t* __restrict__ X, int64_t ld, int n,
                                                  const int64_t* __restrict__ w, const int64_t* __restrict__ b) {
    __shared__ u128 sh[NT / 32];
    __shared__ int64_t s_isq;
    __shared__ int s_zero;
    int64_t* x = X + (int64_t)blockIdx.x * ld;
    u128 s = 0;
    for (int j = threadIdx.x; j < n; j += NT) s += (u128)(i128)x[j];
    s = block_sum_u128(s, sh);
    int64_t mean = lo64((i128)s / (i128)n);
    u128 ss = 0;
    for (int j = threadIdx.x; j < n; j += NT) {
        int64_t dl = wsub(x[j], mean);
        ss += (u128)((i128)dl * dl);
    }
    ss = block_sum_u128(ss, sh);
    if (threadIdx.x == 0) {
        i128 var = (i128)ss / (i128)n;
        s_zero = var <= 0;
        int64_t isq = var > 0 ? isqrt_u128((u128)var) : 0;
        s_isq = isq == 0 ? 1 : isq;
    }
    __syncthreads();
    if (s_zero) {
        for (int j = threadIdx.x; j < n; j += NT) x[j] = b[j];
        return;
    }
    const int64_t isq = s_isq;
    const double rd = 1.0 / (double)isq;
    for (int j = threadIdx.x; j < n; j += NT) {
        const int64_t dl = wsub(x[j], mean), wj = w[j];
        x[j] = wadd(muldiv_trunc(dl, wj, d_i64(wj), isq, rd), b[j]);
    }
}

// NormalizeRow with one warp per row and the row held in registers (n <= 32 * PER): the two Int128
// sums reduce by shuffles, every lane takes the same mean / variance / square root, no block barrier.
// floor(v / n) for v < 2^128 and 1 <= n < 2^32 by long division over 32-bit limbs: each step
// divides (r << 32 | limb) < n * 2^32 with inv = floor((2^64 - 1) / n), an estimate at most two
// below the quotient.
SLX_DEV u128 udiv128_u32(u128 v, uint32_t n, uint64_t inv) {
    u128 q = 0;
    uint64_t r = 0;
#pragma unroll
    for (int i = 3; i >= 0; i--) {
        const uint64_t cur = (r << 32) | (uint64_t)(uint32_t)(v >> (32 * i));
        uint64_t qi = __umul64hi(cur, inv);
        r = cur - qi * n;
        while (r >= n) { qi++; r -= n; }
        q |= (u128)qi << (32 * i);
    }
    return q;
}

// (long)((Int128)s / n), truncating toward zero
SLX_DEV int64_t div_i128_n(u128 s, uint32_t n, uint64_t inv) {
    const bool neg = (i128)s < 0;
    const u128 q = udiv128_u32(neg ? (u128)0 - s : s, n, inv);
    return lo64(neg ? -(i128)q : (i128)q);
}

template <int PER>
__global__ __launch_bounds__(256, 4) void k_layernorm_warp(int64_t* __restrict__ X, int64_t ld, int rows, int n,
                                                         const int64_t* __restrict__ w, const int64_t* __restrict__ b) {
    __shared__ int64_t sw[32 * PER], sb[32 * PER];  // the row's weight and bias, staged once per block
    __shared__ double swd[32 * PER];                 // the weight as a double (exact below 2^51)
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        sw[j] = w[j];
        sb[j] = b[j];
        swd[j] = d_i64(w[j]);
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const uint64_t inv = ~0ULL / (uint64_t)n;
    for (int row = blockIdx.x * 8 + (threadIdx.x >> 5); row < rows; row += gridDim.x * 8) {
        int64_t* x = X + (int64_t)row * ld;
        int64_t v[PER];
        u128 s = 0;
#pragma unroll
        for (int i = 0; i < PER; i++) {
            const int j = lane + 32 * i;
            v[i] = j < n ? __ldcs(x + j) : 0;
            s += (u128)(i128)v[i];
        }
        s = warp_sum_u128(s);
        const int64_t mean = div_i128_n(s, (uint32_t)n, inv);
        u128 ss = 0;
#pragma unroll
        for (int i = 0; i < PER; i++) {
            if (lane + 32 * i < n) {
                v[i] = wsub(v[i], mean);
                ss += (u128)((i128)v[i] * v[i]);
            }
        }
        ss = warp_sum_u128(ss);
        // Int128 variance = sumSq / n (a wrapped, negative sumSq gives var <= 0 as in the reference)
        const i128 var = (i128)ss < 0 ? (i128)0 : (i128)udiv128_u32(ss, (uint32_t)n, inv);
        if (var <= 0) {
#pragma unroll
            for (int i = 0; i < PER; i++)
                if (lane + 32 * i < n) x[lane + 32 * i] = sb[lane + 32 * i];
            continue;
        }
        int64_t isq = isqrt_u128((u128)var);
        if (isq == 0) isq = 1;
        const double rd = 1.0 / (double)isq;
#pragma unroll
        for (int i = 0; i < PER; i++) {
            const int j = lane + 32 * i;
            if (j < n) __stcs(x + j, wadd(muldiv_trunc(v[i], sw[j], swd[j], isq, rd), sb[j]));
        }
    }
}

// NormalizeRow again, for rows whose length n is a multiple of 4, with each lane taking four
// consecutive values at a time (columns 128 q + 4 lane + 0..3): the row is read three times (sum,
// sum of squares, output; the rereads come from cache) instead of being held in registers, so the
// kernel needs few registers and keeps many rows in flight. With planes given it also writes the
// outputs' five balanced digit planes ([5][Mpad][Kpad] int8, the next projection's activation
// operand; columns n..Kpad zero) and raises *overflow for a value beyond five digits.
template <int NQ>
__global__ __launch_bounds__(256) void k_layernorm_q(int64_t* __restrict__ X, int64_t ld, int rows, int n,
                                                     const int64_t* __restrict__ w, const int64_t* __restrict__ b,
                                                     int Mpad, int Kpad, int8_t* __restrict__ planes, int* overflow) {
    const int lane = threadIdx.x & 31;
    const uint64_t inv = ~0ULL / (uint64_t)n;
    bool bad = false;
    for (int row = blockIdx.x * 8 + (threadIdx.x >> 5); row < rows; row += gridDim.x * 8) {
        int64_t* x = X + (int64_t)row * ld;
        // one pass for the sum and the sum of squares; with every |x| < 2^62 no x - mean wraps, and
        // then sum (x - mean)^2 = Q - 2 mean S + n mean^2 holds exactly in wrapping 128-bit arithmetic
        u128 s = 0, sq = 0;
        bool wide = false;
#pragma unroll
        for (int q = 0; q < NQ; q++) {
            const int j = 128 * q + 4 * lane;
            if (j < n) {
                const longlong2 a = __ldg((const longlong2*)(x + j)), c = __ldg((const longlong2*)(x + j + 2));
                s += (u128)(i128)a.x + (u128)(i128)a.y + (u128)(i128)c.x + (u128)(i128)c.y;
                sq += (u128)((i128)a.x * a.x) + (u128)((i128)a.y * a.y) + (u128)((i128)c.x * c.x) + (u128)((i128)c.y * c.y);
                wide |= (((uint64_t)a.x + (1ULL << 62)) | ((uint64_t)a.y + (1ULL << 62)) | ((uint64_t)c.x + (1ULL << 62)) |
                         ((uint64_t)c.y + (1ULL << 62))) >> 63;
            }
        }
        s = warp_sum_u128(s);
        sq = warp_sum_u128(sq);
        const int64_t mean = div_i128_n(s, (uint32_t)n, inv);
        u128 ss;
        if (!__any_sync(0xffffffffu, wide)) {
            const uint64_t s_lo = (uint64_t)s, s_hi = (uint64_t)(s >> 64);
            const u128 ms = (u128)((i128)mean * (int64_t)s_lo) + ((u128)(s_lo >> 63) * (u128)(uint64_t)mean << 64) +
                            ((u128)((uint64_t)mean * s_hi) << 64);  // mean * S mod 2^128
            ss = sq - 2 * ms + (u128)n * (u128)((i128)mean * mean);
        } else {  // values near the int64 limits: the reference's wrapping differences, a second pass
            ss = 0;
#pragma unroll
            for (int q = 0; q < NQ; q++) {
                const int j = 128 * q + 4 * lane;
                if (j < n) {
                    const longlong2 a = __ldg((const longlong2*)(x + j)), c = __ldg((const longlong2*)(x + j + 2));
                    const int64_t d0 = wsub(a.x, mean), d1 = wsub(a.y, mean), d2 = wsub(c.x, mean), d3 = wsub(c.y, mean);
                    ss += (u128)((i128)d0 * d0) + (u128)((i128)d1 * d1) + (u128)((i128)d2 * d2) + (u128)((i128)d3 * d3);
                }
            }
            ss = warp_sum_u128(ss);
        }
        // Int128 variance = sumSq / n (a wrapped, negative sumSq gives var <= 0 as in the reference)
        const i128 var = (i128)ss < 0 ? (i128)0 : (i128)udiv128_u32(ss, (uint32_t)n, inv);
        int64_t isq = var > 0 ? isqrt_u128((u128)var) : 1;
        if (isq == 0) isq = 1;
        const double rd = 1.0 / (double)isq;
#pragma unroll 1
        for (int q = 0; q < NQ; q++) {  // not unrolled: the per-value division code stays in the instruction cache
            const int j = 128 * q + 4 * lane;
            int64_t y[4] = {0, 0, 0, 0};
            if (j < n) {
                // the weight and bias (the same for every row: cached reads)
                const longlong2 b0 = __ldg((const longlong2*)(b + j)), b1 = __ldg((const longlong2*)(b + j + 2));
                const int64_t bb[4] = {b0.x, b0.y, b1.x, b1.y};
                if (var <= 0) {  // x = bias (IntegerLayerNorm.cs:39-44)
#pragma unroll
                    for (int e = 0; e < 4; e++) y[e] = bb[e];
                } else {
                    const longlong2 a = __ldg((const longlong2*)(x + j)), c = __ldg((const longlong2*)(x + j + 2));
                    const longlong2 w0 = __ldg((const longlong2*)(w + j)), w1 = __ldg((const longlong2*)(w + j + 2));
                    const int64_t v[4] = {a.x, a.y, c.x, c.y}, ww[4] = {w0.x, w0.y, w1.x, w1.y};
#pragma unroll
                    for (int e = 0; e < 4; e++)
                        y[e] = wadd(muldiv_trunc(wsub(v[e], mean), ww[e], d_i64(ww[e]), isq, rd), bb[e]);
                }
                *(longlong2*)(x + j) = make_longlong2(y[0], y[1]);
                *(longlong2*)(x + j + 2) = make_longlong2(y[2], y[3]);
            }
            if (planes && j < Kpad) {
                uint32_t wd[5];
                digit_words4(y[0], y[1], y[2], y[3], wd, bad);
#pragma unroll
                for (int i = 0; i < 5; i++) *(uint32_t*)(planes + ((int64_t)i * Mpad + row) * Kpad + j) = wd[i];
            }
        }
    }
    if (bad) atomicOr(overflow, 1);
}

// RmsNormRow (IntegerLayerNorm.cs:71-93); row r = segment (r % per) of line (r / per).
__global__ __launch_bounds__(NT) void k_rmsnorm(int64_t* __restrict__ X, int64_t ld, int per, int n,
                                                const int64_t* __restrict__ w) {
    __shared__ u128 sh[NT / 32];
    __shared__ int64_t s_rms;
    __shared__ int s_skip;
    int r = blockIdx.x;
    int64_t* x = X + (int64_t)(r / per) * ld + (int64_t)(r % per) * n;
    u128 ss = 0;
    for (int j = threadIdx.x; j < n; j += NT) ss += (u128)((i128)x[j] * x[j]);
    ss = block_sum_u128(ss, sh);
    if (threadIdx.x == 0) {
        i128 ms = (i128)ss / (i128)n;
        s_skip = ms <= 0;
        int64_t rms = ms > 0 ? isqrt_u128((u128)ms) : 0;
        s_rms = rms == 0 ? 1 : rms;
    }
    __syncthreads();
    if (s_skip) return;
    const int64_t rms = s_rms;
    const double rd = 1.0 / (double)rms;
    for (int j = threadIdx.x; j < n; j += NT) {
        const int64_t wj = w[j];
        x[j] = muldiv_trunc(x[j], wj, d_i64(wj), rms, rd);
    }
}

// RmsNormRow for short rows (n <= 32 * PL, e.g. RmsNormPerHead's head segments): one warp per row,
// the lane's values in registers, the Int128 sum reduced by shuffles, every lane taking the same
// square root; row r is segment (r % per) of line (r / per).
template <int PL>
__global__ __launch_bounds__(256) void k_rmsnorm_warp(int64_t* __restrict__ X, int64_t ld, int per, int n, int rows,
                                                      const int64_t* __restrict__ w) {
    const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= rows) return;
    int64_t* x = X + (int64_t)(r / per) * ld + (int64_t)(r % per) * n;
    int64_t v[PL];
    u128 ss = 0;
#pragma unroll
    for (int e = 0; e < PL; e++) {
        const int j = lane + 32 * e;
        v[e] = j < n ? x[j] : 0;
        ss += (u128)((i128)v[e] * v[e]);
    }
    ss = warp_sum_u128(ss);
    if ((i128)ss < (i128)n) return;  // ms = sumSq / n <= 0: the row is left as it is
    int64_t rms = isqrt_u128(udiv128_u32(ss, (uint32_t)n, ~0ULL / (uint32_t)n));
    if (rms == 0) rms = 1;
    const double rd = 1.0 / (double)rms;
#pragma unroll
    for (int e = 0; e < PL; e++) {
        const int j = lane + 32 * e;
        if (j < n) {
            const int64_t wj = w[j];
            x[j] = muldiv_trunc(v[e], wj, d_i64(wj), rms, rd);
        }
    }
}

// The causal block's norms around a residual add, one block per row of n = 256 * EPT (EPT
// consecutive values a thread, kept in registers between the steps):
//   with w1:  y <- RmsNormRow(y; w1) + r   (the post-attention / post-FFN norm and the residual add)
//   with w2:  z <- RmsNormRow(y; w2)       (the next pre-norm), with, when planes is given, z's five
//             balanced digit planes [5][Mpad][Kpad] for the projections that read it (*overflow raised
//             for a value beyond five digits).
// RmsNormRow (IntegerLayerNorm.cs:71-93): ms = (Int128 sum x^2) / n; a row with ms <= 0 is left as it
// is; otherwise x = (long)((Int128)x * w / max(ISqrt(ms), 1)).
SLX_DEV int64_t rms_of_block(u128 ss, int n, u128* sh, bool& skip) {
    ss = warp_sum_u128(ss);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = ss;
    __syncthreads();
    u128 t = 0;
#pragma unroll
    for (int i = 0; i < NT / 32; i++) t += sh[i];  // every thread forms the same total
    // ms = (Int128)t / n is at most 0 exactly when t (signed) < n; otherwise t > 0 and the unsigned
    // division by the 32-bit n is the same quotient
    skip = (i128)t < (i128)n;
    const int64_t r = skip ? 0 : isqrt_u128(udiv128_u32(t, (uint32_t)n, ~0ULL / (uint32_t)n));
    return r == 0 ? 1 : r;
}

template <int EPT>
__global__ __launch_bounds__(NT) void k_rms_pair(int64_t* __restrict__ Y, const int64_t* __restrict__ R,
                                                 int64_t* __restrict__ Z, int n, const int64_t* __restrict__ w1,
                                                 const int64_t* __restrict__ w2, int Mpad, int Kpad,
                                                 int8_t* __restrict__ planes, int* overflow) {
    __shared__ u128 sh1[NT / 32], sh2[NT / 32];
    const int64_t row = blockIdx.x;
    const int j0 = threadIdx.x * EPT;
    const bool in = j0 < n;
    int64_t v[EPT];
#pragma unroll
    for (int e = 0; e < EPT; e += 2) {
        const longlong2 a = in ? *(const longlong2*)(Y + row * n + j0 + e) : make_longlong2(0, 0);
        v[e] = a.x;
        v[e + 1] = a.y;
    }
    if (w1) {
        u128 ss = 0;
#pragma unroll
        for (int e = 0; e < EPT; e++) ss += (u128)((i128)v[e] * v[e]);
        bool skip;
        const int64_t rms = rms_of_block(ss, n, sh1, skip);
        const double rd = 1.0 / (double)rms;
        if (in) {
#pragma unroll
            for (int e = 0; e < EPT; e += 2) {
                const longlong2 r = *(const longlong2*)(R + row * n + j0 + e);
                if (!skip) {
                    const longlong2 w = *(const longlong2*)(w1 + j0 + e);
                    v[e] = muldiv_trunc(v[e], w.x, d_i64(w.x), rms, rd);
                    v[e + 1] = muldiv_trunc(v[e + 1], w.y, d_i64(w.y), rms, rd);
                }
                v[e] = wadd(v[e], r.x);
                v[e + 1] = wadd(v[e + 1], r.y);
                *(longlong2*)(Y + row * n + j0 + e) = make_longlong2(v[e], v[e + 1]);
            }
        }
    }
    if (!w2) return;
    u128 ss = 0;
#pragma unroll
    for (int e = 0; e < EPT; e++) ss += (u128)((i128)v[e] * v[e]);
    bool skip;
    const int64_t rms = rms_of_block(ss, n, sh2, skip);
    const double rd = 1.0 / (double)rms;
    if (!in) return;
    bool bad = false;
#pragma unroll
    for (int e = 0; e < EPT; e += 4) {
        int64_t z[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            z[u] = v[e + u];
            if (!skip) {
                const int64_t w = w2[j0 + e + u];
                z[u] = muldiv_trunc(z[u], w, d_i64(w), rms, rd);
            }
        }
        *(longlong2*)(Z + row * n + j0 + e) = make_longlong2(z[0], z[1]);
        *(longlong2*)(Z + row * n + j0 + e + 2) = make_longlong2(z[2], z[3]);
        if (planes) {
            uint32_t wd[5];
            digit_words4(z[0], z[1], z[2], z[3], wd, bad);
#pragma unroll
            for (int i = 0; i < 5; i++) *(uint32_t*)(planes + ((int64_t)i * Mpad + row) * Kpad + j0 + e) = wd[i];
        }
    }
    if (bad) atomicOr(overflow, 1);
}
}  // namespace

int layernorm_rows(int64_t* x, int64_t ld, int rows, int n, const int64_t* w, const int64_t* b, cudaStream_t st) {
    if (rows <= 0) return 0;
    const unsigned wb = (unsigned)std::min((rows + 7) / 8, 148 * 4);  // four blocks per SM
    if (n <= 256) k_layernorm_warp<8><<<wb, 256, 0, st>>>(x, ld, rows, n, w, b);
    else if (n <= 512) k_layernorm_warp<16><<<wb, 256, 0, st>>>(x, ld, rows, n, w, b);
    else if (n <= 768) k_layernorm_warp<24><<<wb, 256, 0, st>>>(x, ld, rows, n, w, b);
    else if (n <= 1024) k_layernorm_warp<32><<<wb, 256, 0, st>>>(x, ld, rows, n, w, b);
    else k_layernorm<<<rows, NT, 0, st>>>(x, ld, n, w, b);
    return 1;
}

int layernorm_rows_digits(int64_t* x, int64_t ld, int rows, int n, const int64_t* w, const int64_t* b, int64_t Mpad,
                          int64_t Kpad, int8_t* planes, int* overflow, cudaStream_t st) {
    if (rows <= 0) return 0;
    const int nq = (int)((Kpad + 127) / 128);
    if (n % 4 != 0 || (ld & 1) != 0 || ((uintptr_t)x & 15) != 0 || ((uintptr_t)w & 15) != 0 || ((uintptr_t)b & 15) != 0 ||
        nq > 8 || Kpad % 128 != 0 || Kpad < n)
        return -1;
    int k = 0;
    if (planes && Mpad > rows)  // padding rows of every plane: zero digits
        for (int i = 0; i < 5; i++, k++)
            cudaMemsetAsync(planes + ((int64_t)i * Mpad + rows) * Kpad, 0, (size_t)(Mpad - rows) * Kpad, st);
    const unsigned wb = (unsigned)std::min((rows + 7) / 8, 148 * 8);
    switch (nq) {
        case 1: k_layernorm_q<1><<<wb, 256, 0, st>>>(x, ld, rows, n, w, b, (int)Mpad, (int)Kpad, planes, overflow); break;
        case 2: k_layernorm_q<2><<<wb, 256, 0, st>>>(x, ld, rows, n, w, b, (int)Mpad, (int)Kpad, planes, overflow); break;
        case 3: case 4: k_layernorm_q<4><<<wb, 256, 0, st>>>(x, ld, rows, n, w, b, (int)Mpad, (int)Kpad, planes, overflow); break;
        case 5: case 6: k_layernorm_q<6><<<wb, 256, 0, st>>>(x, ld, rows, n, w, b, (int)Mpad, (int)Kpad, planes, overflow); break;
        default: k_layernorm_q<8><<<wb, 256, 0, st>>>(x, ld, rows, n, w, b, (int)Mpad, (int)Kpad, planes, overflow); break;
    }
    return k + 1;
}

int rmsnorm_rows(int64_t* x, int64_t ld, int rows, int per, int n, const int64_t* w, cudaStream_t st) {
    if (rows <= 0) return 0;
    const unsigned wb = (unsigned)((rows + 7) / 8);
    if (n <= 32) k_rmsnorm_warp<1><<<wb, 256, 0, st>>>(x, ld, per, n, rows, w);
    else if (n <= 64) k_rmsnorm_warp<2><<<wb, 256, 0, st>>>(x, ld, per, n, rows, w);
    else if (n <= 128) k_rmsnorm_warp<4><<<wb, 256, 0, st>>>(x, ld, per, n, rows, w);
    else if (n <= 256) k_rmsnorm_warp<8><<<wb, 256, 0, st>>>(x, ld, per, n, rows, w);
    else if (n <= 512) k_rmsnorm_warp<16><<<wb, 256, 0, st>>>(x, ld, per, n, rows, w);
    else k_rmsnorm<<<rows, NT, 0, st>>>(x, ld, per, n, w);
    return 1;
}

int rms_pair_rows(int64_t* y, const int64_t* r, int64_t* z, int rows, int n, const int64_t* w1, const int64_t* w2,
                  int64_t Mpad, int64_t Kpad, int8_t* planes, int* overflow, cudaStream_t st) {
    if (rows <= 0) return 0;
    if (n % (4 * NT) != 0 || n > 16 * NT || ((uintptr_t)y & 15) || (r && ((uintptr_t)r & 15)) || ((uintptr_t)z & 15) ||
        (w1 && ((uintptr_t)w1 & 15)) || (planes && (Kpad != n || Mpad < rows)))
        return -1;
    int k = 0;
    if (planes && Mpad > rows)  // padding rows of every plane: zero digits
        for (int i = 0; i < 5; i++, k++)
            cudaMemsetAsync(planes + ((int64_t)i * Mpad + rows) * Kpad, 0, (size_t)(Mpad - rows) * Kpad, st);
    switch (n / NT) {
        case 4: k_rms_pair<4><<<rows, NT, 0, st>>>(y, r, z, n, w1, w2, (int)Mpad, (int)Kpad, planes, overflow); break;
        case 8: k_rms_pair<8><<<rows, NT, 0, st>>>(y, r, z, n, w1, w2, (int)Mpad, (int)Kpad, planes, overflow); break;
        case 12: k_rms_pair<12><<<rows, NT, 0, st>>>(y, r, z, n, w1, w2, (int)Mpad, (int)Kpad, planes, overflow); break;
        default: k_rms_pair<16><<<rows, NT, 0, st>>>(y, r, z, n, w1, w2, (int)Mpad, (int)Kpad, planes, overflow); break;
    }
    return k + 1;
}

// ------------------------------------------------------------------------------------------
// RoPE (IntegerAttention.ApplyRoPE, IntegerAttention.cs:35-58)
// ------------------------------------------------------------------------------------------
namespace {
// With only_if, nothing is done unless *only_if is nonzero (the rotation is then needed by the exact
// attention kernel, the tensor-core path having rotated only its digit planes).
__global__ void k_rope(int64_t* __restrict__ X, int64_t ld, int T, int nh, int hd, const int64_t* __restrict__ cs,
                       const int64_t* __restrict__ sn, int64_t total, const int* __restrict__ only_if) {
    if (only_if && *only_if == 0) return;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    int half = hd / 2;
    int p = (int)(i % half);
    int64_t mh = i / half;
    int h = (int)(mh % nh);
    int64_t m = mh / nh;
    int t = (int)(m % T);
    int64_t* hb = X + m * ld + (int64_t)h * hd;
    int64_t c = cs[(int64_t)t * half + p], s = sn[(int64_t)t * half + p];
    int64_t x0 = hb[p], x1 = hb[p + half];
    hb[p] = lo64(sar128((i128)((u128)((i128)x0 * c) - (u128)((i128)x1 * s)), 30));
    hb[p + half] = lo64(sar128((i128)((u128)((i128)x0 * s) + (u128)((i128)x1 * c)), 30));
    }
}
}  // namespace

int rope_rows(int64_t* x, int64_t ld, int B, int T, int nh, int hd, const int64_t* cos, const int64_t* sin,
               cudaStream_t st, const int* only_if) {
    int64_t total = (int64_t)B * T * nh * (hd / 2);
    if (total <= 0) return 0;
    // gated: it usually does nothing, so a small grid strides over the pairs
    const int64_t grid = only_if ? std::min<int64_t>((total + 255) / 256, 148 * 2) : (total + 255) / 256;
    k_rope<<<(unsigned)grid, 256, 0, st>>>(x, ld, T, nh, hd, cos, sin, total, only_if);
    return 1;
}

// ------------------------------------------------------------------------------------------
// Attention, one warp per query row (IntegerAttention.cs:60-109, 165-202, 246-289, 333-377):
// scores (long)(dot >> shift) / ISqrt64(hd) with masked slots set to -2^29, FixedSoftmax over the
// whole row, then out[d] += (long)((Int128)w * v[s][d] >> 30) term by term.
// ------------------------------------------------------------------------------------------
namespace {
constexpr int AW = 4;  // warps (query rows) per block

__global__ __launch_bounds__(AW * 32) void k_attention(const int64_t* __restrict__ Q, int64_t ldq,
                                                       const int64_t* __restrict__ Kp, int64_t ldk,
                                                       const int64_t* __restrict__ V, int64_t ldv,
                                                       int64_t* __restrict__ O, int64_t ldo, int T, int nh, int nkv,
                                                       int hd, int score_shift, int64_t sqrt_hd, int mode,
                                                       int window, int B, const int* __restrict__ only_if) {
    if (only_if && *only_if == 0) return;
    extern __shared__ int64_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nxb = (T + AW - 1) / AW;
    const int64_t nblocks = (int64_t)nxb * nh * B;
    for (int64_t blk = blockIdx.x; blk < nblocks; blk += gridDim.x) {
    const int t = (int)(blk % nxb) * AW + warp;
    const int h = (int)((blk / nxb) % nh), b = (int)(blk / ((int64_t)nxb * nh));
    int64_t* sc = smem + (size_t)warp * (T + hd);
    int64_t* qrow = sc + T;
    if (t >= T) continue;
    const int kvh = h / (nh / nkv);
    const int64_t rowq = (int64_t)b * T + t;
    for (int d = lane; d < hd; d += 32) qrow[d] = Q[rowq * ldq + (int64_t)h * hd + d];
    __syncwarp();
    const int64_t mask = -(1LL << 29);
    const int ws = t - window + 1 > 0 ? t - window + 1 : 0;
    int64_t mx = INT64_MIN;
    for (int s = lane; s < T; s += 32) {
        int64_t v;
        if ((mode >= 1 && s > t) || (mode == 2 && s < ws)) {
            v = mask;
        } else {
            const int64_t* kr = Kp + ((int64_t)b * T + s) * ldk + (int64_t)kvh * hd;
            u128 acc = 0;
            for (int d = 0; d < hd; d++) acc += (u128)((i128)qrow[d] * kr[d]);
            v = cs_div64(lo64(sar128((i128)acc, score_shift)), sqrt_hd);
        }
        sc[s] = v;
        mx = v > mx ? v : mx;
    }
    mx = warp_max_i64(mx);
    u128 sum = 0;
    for (int s = lane; s < T; s += 32) {
        int64_t e = fixed_exp30(wsub(sc[s], mx));
        sc[s] = e;
        sum += (u128)(i128)e;
    }
    sum = warp_sum_u128(sum);
    const i128 ssum = (i128)sum;
    const bool fast = ssum > 0 && (sum >> 64) == 0;
    for (int s = lane; s < T; s += 32) {
        int64_t e = sc[s];
        int64_t p;
        if (ssum == 0)
            p = (1LL << 30) / T;
        else if (fast && e >= 0 && e <= (1LL << 33))
            p = (int64_t)(((uint64_t)e << 30) / (uint64_t)sum);
        else
            p = lo64(((i128)e * (1LL << 30)) / ssum);
        sc[s] = p;
    }
    __syncwarp();
    int64_t* orow = O + rowq * ldo + (int64_t)h * hd;
    const int64_t* vb = V + (int64_t)b * T * ldv + (int64_t)kvh * hd;
    for (int d = lane; d < hd; d += 32) {
        int64_t acc = 0;
        for (int s = 0; s < T; s++) acc = wadd(acc, lo64(sar128((i128)sc[s] * vb[(int64_t)s * ldv + d], 30)));
        orow[d] = acc;
    }
    __syncwarp();  // the next query row reuses this warp's scores
    }
}
}  // namespace

int attention(const int64_t* q, int64_t ldq, const int64_t* k, int64_t ldk, const int64_t* v, int64_t ldv,
               int64_t* out, int64_t ldo, int B, int T, int nh, int nkv, int hd, int score_shift, int64_t sqrt_hd,
               int mode, int window, cudaStream_t st, const int* only_if) {
    if (B * T <= 0) return 0;
    size_t smem = (size_t)AW * (T + hd) * sizeof(int64_t);
    slx::ensure_smem((const void*)k_attention, smem);
    const int64_t nblocks = (int64_t)((T + AW - 1) / AW) * nh * B;
    const int64_t grid = only_if ? std::min<int64_t>(nblocks, 4 * 148) : nblocks;
    k_attention<<<(unsigned)grid, AW * 32, smem, st>>>(q, ldq, k, ldk, v, ldv, out, ldo, T, nh, nkv, hd, score_shift,
                                                      sqrt_hd, mode, window, B, only_if);
    return 1;
}

// ------------------------------------------------------------------------------------------
// FFN gate, residual adds, pooling
// ------------------------------------------------------------------------------------------
namespace {
// IntegerFFN.Apply: up[i] = (long)((Int128)FixedSiLU(gate[i]) * up[i] >> 30) (IntegerFFN.cs:84-89)
__global__ void k_silu_gate(const int64_t* __restrict__ G, int64_t ldg, int64_t* __restrict__ U, int64_t ldu, int F,
                            int rows) {
    const int f = blockIdx.x * blockDim.x + threadIdx.x;
    if (f >= F) return;
    for (int m = blockIdx.y; m < rows; m += gridDim.y) {
        int64_t* u = U + (int64_t)m * ldu + f;
        *u = silu_gate30(G[(int64_t)m * ldg + f], *u);
    }
}

// The same gate for four consecutive columns a thread, which also writes the five balanced digit
// planes of the gated values ([5][Mpad][Kpad] int8, the next projection's activation operand) and sets
// *overflow when a value needs a sixth digit. Columns F..Kpad get zero digits; rows M..Mpad are left
// to the caller. F % 4 == 0 and 16-byte aligned rows.
__global__ void k_silu_gate_digits(const int64_t* __restrict__ G, int64_t ldg, int64_t* __restrict__ U, int64_t ldu,
                                   int F, int rows, int Mpad, int Kpad, int8_t* __restrict__ planes, int* overflow) {
    const int f = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
    if (f >= Kpad) return;
    bool bad = false;
    for (int m = blockIdx.y; m < rows; m += gridDim.y) {
        int64_t y[4] = {0, 0, 0, 0};
        if (f < F) {
            const int64_t* g = G + (int64_t)m * ldg + f;
            int64_t* u = U + (int64_t)m * ldu + f;
            const longlong2 g0 = *(const longlong2*)g, g1 = *(const longlong2*)(g + 2);
            const longlong2 u0 = *(const longlong2*)u, u1 = *(const longlong2*)(u + 2);
            y[0] = silu_gate30(g0.x, u0.x);
            y[1] = silu_gate30(g0.y, u0.y);
            y[2] = silu_gate30(g1.x, u1.x);
            y[3] = silu_gate30(g1.y, u1.y);
            *(longlong2*)u = make_longlong2(y[0], y[1]);
            *(longlong2*)(u + 2) = make_longlong2(y[2], y[3]);
        }
        uint32_t w[5];
        digit_words4(y[0], y[1], y[2], y[3], w, bad);
#pragma unroll
        for (int i = 0; i < 5; i++) *(uint32_t*)(planes + ((int64_t)i * Mpad + m) * Kpad + f) = w[i];
    }
    if (bad) atomicOr(overflow, 1);
}

__global__ void k_add(int64_t* __restrict__ D, int64_t ldd, const int64_t* __restrict__ S, int64_t lds, int n,
                      int64_t total) {
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= total) return;
    int64_t m = i / n, j = i % n;
    D[m * ldd + j] = wadd(D[m * ldd + j], S[m * lds + j]);
}

// MeanPool (IntegerTransformerSource.Forward.cs:69-87)
// A block owns 32 columns of one sequence; its eight warps sum interleaved rows (a warp reads 256
// contiguous bytes of a row) and the Int128 partials are added in shared memory.
constexpr int MP_COLS = 32, MP_GROUPS = 8;
__global__ __launch_bounds__(MP_COLS * MP_GROUPS) void k_mean_pool(const int64_t* __restrict__ X, int64_t ld, int T,
                                                                   int d, int64_t* __restrict__ P) {
    __shared__ u128 part[MP_GROUPS][MP_COLS];
    const int c = threadIdx.x % MP_COLS, g = threadIdx.x / MP_COLS;
    const int j = blockIdx.x * MP_COLS + c, b = blockIdx.y;
    u128 s = 0;
    if (j < d)
        for (int t = g; t < T; t += MP_GROUPS) s += (u128)(i128)X[((int64_t)b * T + t) * ld + j];
    part[g][c] = s;
    __syncthreads();
    if (g == 0 && j < d) {
        for (int i = 1; i < MP_GROUPS; i++) s += part[i][c];
        P[(int64_t)b * d + j] = T > 0 ? lo64((i128)s / (i128)T) : 0;
    }
}

__global__ void k_gather_last(const int64_t* __restrict__ X, int64_t ld, int T, int d, int64_t* __restrict__ D) {
    int j = blockIdx.x * blockDim.x + threadIdx.x, b = blockIdx.y;
    if (j < d) D[(int64_t)b * d + j] = X[((int64_t)b * T + T - 1) * ld + j];
}

// VocabLattice.ArgmaxBruteForce (Lattice/VocabLattice.cs:103-126): h[j] = (float)(last[j] * 2^-s)
// (IntegerCausalSource.ForwardCausalFloat :114-122), dot accumulated in order j = 0..d-1 with
// separate fp32 multiply and add, strict '>' (first maximum wins, NaN and -inf never selected).
// A block owns AR vocabulary rows (one per thread) and up to AQ queries. Components stream in
// chunks of AC: the block stages its rows' (float)(Half) values (coalesced block reads, converted
// once for all its queries) and the queries' floats in shared memory, then every thread extends
// its AQ independent dot chains by the chunk. Components past d are staged as zeros on both sides:
// adding the +0 product leaves every chain unchanged (a chain that starts at +0 is never -0).
// Candidates are combined through a 64-bit key: ordered score bits, then the inverted row id.
constexpr int AR = 128, AQ = 16, AC = 64, APAD = AC + 4;
SLX_DEV uint32_t ordered(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Eight consecutive elements e0..e0+7 (e0 a multiple of 8) of a GGUF tensor as (float)(Half), with
// the block scale read once for Q8_0 / Q4_0; elements of blocks past nblocks are 0 (dequant_elem).
// Small integers become floats exactly by the 2^23 bias: float(2^23 + n) - (2^23 + c) = n - c.
SLX_DEV float2 half_round2(float a, float b) { return __half22float2(__floats2half2_rn(a, b)); }
template <int DT>
SLX_DEV void dequant8_half(const uint8_t* __restrict__ base, int64_t e0, int64_t nblocks, float* out) {
    if constexpr (DT == DT_Q4_0 || DT == DT_Q8_0) {
        const int64_t b = e0 >> 5;
        if (b >= nblocks) {
#pragma unroll
            for (int t = 0; t < 8; t++) out[t] = 0.0f;
            return;
        }
        if constexpr (DT == DT_Q4_0) {
            const uint8_t* blk = base + b * 18;
            const float sc = h2f(ld_u16(blk));
            const uint16_t* q = (const uint16_t*)(blk + 2 + ((e0 & 31) >> 1));  // element 2j: low nibble of byte j
            const uint32_t w = (uint32_t)q[0] | ((uint32_t)q[1] << 16);
#pragma unroll
            for (int t = 0; t < 8; t += 2) {
                const float x0 = __fsub_rn(__uint_as_float(0x4B000000u | ((w >> (4 * t)) & 15u)), 8388616.0f);
                const float x1 = __fsub_rn(__uint_as_float(0x4B000000u | ((w >> (4 * t + 4)) & 15u)), 8388616.0f);
                const float2 r = half_round2(__fmul_rn(sc, x0), __fmul_rn(sc, x1));
                out[t] = r.x;
                out[t + 1] = r.y;
            }
        } else {
            const uint8_t* blk = base + b * 34;
            const float sc = h2f(ld_u16(blk));
            const uint16_t* q = (const uint16_t*)(blk + 2 + (e0 & 31));
#pragma unroll
            for (int t = 0; t < 4; t++) {
                const uint32_t pr = q[t];
                const float x0 = __fsub_rn(__uint_as_float(0x4B000000u | ((pr & 0xFFu) ^ 0x80u)), 8388736.0f);
                const float x1 = __fsub_rn(__uint_as_float(0x4B000000u | ((pr >> 8) ^ 0x80u)), 8388736.0f);
                const float2 r = half_round2(__fmul_rn(sc, x0), __fmul_rn(sc, x1));
                out[2 * t] = r.x;
                out[2 * t + 1] = r.y;
            }
        }
    } else {
#pragma unroll
        for (int t = 0; t < 8; t++) out[t] = h2f(f2h(dequant_elem(DT, base, e0 + t, nblocks)));
    }
}

// NQ queries per block (B rounded up to a power of two, at most AQ): every thread extends NQ
// independent chains per component, so the adds of different queries interleave.
template <int DT, int NQ>
__global__ __launch_bounds__(AR) void k_argmax(const int64_t* __restrict__ last, int B, int d, WDesc tok, int vocab,
                                               double scale, unsigned long long* keys) {
    __shared__ __align__(16) float rows[AR][APAD];
    __shared__ __align__(16) float hs[NQ][AC];
    const int tid = threadIdx.x;
    const int64_t v0 = (int64_t)blockIdx.x * AR;
    const int q0 = blockIdx.y * NQ;
    const int nq = min(NQ, B - q0);
    const bool whole = (d & 7) == 0;  // 8-element groups never straddle a row
    float acc[NQ];
#pragma unroll
    for (int b = 0; b < NQ; b++) acc[b] = 0.0f;
    for (int j0 = 0; j0 < d; j0 += AC) {
        // thread t stages 8-element groups t, t + AR, ... of the [AR][AC] tile (row g / 8, column 8 (g % 8))
#pragma unroll 4
        for (int g = tid; g < AR * AC / 8; g += AR) {
            const int r = g >> 3, c = (g & 7) * 8;
            float e[8];
            if (v0 + r < vocab && j0 + c + 8 <= d && whole) {
                dequant8_half<DT>(tok.data, (v0 + r) * d + j0 + c, tok.nblocks, e);
            } else {
#pragma unroll
                for (int t = 0; t < 8; t++)
                    e[t] = (v0 + r < vocab && j0 + c + t < d)
                               ? h2f(f2h(dequant_elem(DT, tok.data, (v0 + r) * d + j0 + c + t, tok.nblocks)))
                               : 0.0f;
            }
            *reinterpret_cast<float4*>(&rows[r][c]) = make_float4(e[0], e[1], e[2], e[3]);
            *reinterpret_cast<float4*>(&rows[r][c + 4]) = make_float4(e[4], e[5], e[6], e[7]);
        }
        for (int idx = tid; idx < NQ * AC; idx += AR) {
            const int b = idx / AC, c = idx % AC;
            float h = 0.0f;
            if (b < nq && j0 + c < d) h = __double2float_rn((double)last[(int64_t)(q0 + b) * d + j0 + c] * scale);
            hs[b][c] = h;
        }
        __syncthreads();
#pragma unroll 2
        for (int c = 0; c < AC; c += 4) {
            const float4 e = *reinterpret_cast<const float4*>(&rows[tid][c]);
#pragma unroll
            for (int b = 0; b < NQ; b++) {
                const float4 h = *reinterpret_cast<const float4*>(&hs[b][c]);
                float a = acc[b];
                a = __fadd_rn(a, __fmul_rn(h.x, e.x));
                a = __fadd_rn(a, __fmul_rn(h.y, e.y));
                a = __fadd_rn(a, __fmul_rn(h.z, e.z));
                a = __fadd_rn(a, __fmul_rn(h.w, e.w));
                acc[b] = a;
            }
        }
        __syncthreads();
    }
    const int64_t v = v0 + tid;
#pragma unroll
    for (int b = 0; b < NQ; b++) {
        if (b < nq) {
            unsigned long long key = 0;
            if (v < vocab && acc[b] > -INFINITY)
                key = ((unsigned long long)ordered(acc[b]) << 32) | (0xFFFFFFFFu - (uint32_t)v);
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, o);
                key = k2 > key ? k2 : key;
            }
            if ((tid & 31) == 0 && key) atomicMax(keys + q0 + b, key);
        }
    }
}

template <int DT>
void launch_argmax(const int64_t* last, int B, int d, const WDesc& tok, int vocab, double sc, unsigned long long* keys,
                   cudaStream_t st) {
    const unsigned gx = (unsigned)((vocab + AR - 1) / AR);
    if (B == 1) k_argmax<DT, 1><<<dim3(gx, 1), AR, 0, st>>>(last, B, d, tok, vocab, sc, keys);
    else if (B == 2) k_argmax<DT, 2><<<dim3(gx, 1), AR, 0, st>>>(last, B, d, tok, vocab, sc, keys);
    else if (B <= 4) k_argmax<DT, 4><<<dim3(gx, 1), AR, 0, st>>>(last, B, d, tok, vocab, sc, keys);
    else if (B <= 8) k_argmax<DT, 8><<<dim3(gx, 1), AR, 0, st>>>(last, B, d, tok, vocab, sc, keys);
    else k_argmax<DT, AQ><<<dim3(gx, (unsigned)((B + AQ - 1) / AQ)), AR, 0, st>>>(last, B, d, tok, vocab, sc, keys);
}

__global__ void k_keys_to_ids(const unsigned long long* keys, int B, int32_t* ids) {
    int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B) ids[b] = keys[b] ? (int32_t)(0xFFFFFFFFu - (uint32_t)(keys[b] & 0xFFFFFFFFu)) : 0;
}
}  // namespace

int silu_gate(const int64_t* gate, int64_t ldg, int64_t* up, int64_t ldu, int M, int F, cudaStream_t st) {
    if (M <= 0 || F <= 0) return 0;
    const dim3 grid((unsigned)((F + 255) / 256), (unsigned)(M < 65535 ? M : 65535));
    k_silu_gate<<<grid, 256, 0, st>>>(gate, ldg, up, ldu, F, M);
    return 1;
}

int silu_gate_digits(const int64_t* gate, int64_t ldg, int64_t* up, int64_t ldu, int M, int F, int64_t Mpad, int64_t Kpad,
                     int8_t* planes, int* overflow, cudaStream_t st) {
    if (M <= 0 || F <= 0) return 0;
    int n = 0;
    if (Mpad > M)  // padding rows of every plane: zero digits
        for (int i = 0; i < 5; i++, n++)
            cudaMemsetAsync(planes + ((int64_t)i * Mpad + M) * Kpad, 0, (size_t)(Mpad - M) * Kpad, st);
    const dim3 grid((unsigned)((Kpad / 4 + 255) / 256), (unsigned)(M < 65535 ? M : 65535));
    k_silu_gate_digits<<<grid, 256, 0, st>>>(gate, ldg, up, ldu, F, M, (int)Mpad, (int)Kpad, planes, overflow);
    return n + 1;
}

int add_rows(int64_t* dst, int64_t ldd, const int64_t* src, int64_t lds, int M, int n, cudaStream_t st) {
    int64_t total = (int64_t)M * n;
    if (total <= 0) return 0;
    k_add<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(dst, ldd, src, lds, n, total);
    return 1;
}

int mean_pool(const int64_t* x, int64_t ld, int B, int T, int d, int64_t* pooled, cudaStream_t st) {
    if (B <= 0) return 0;
    k_mean_pool<<<dim3((unsigned)((d + MP_COLS - 1) / MP_COLS), (unsigned)B), MP_COLS * MP_GROUPS, 0, st>>>(x, ld, T, d,
                                                                                                     pooled);
    return 1;
}

int gather_last_rows(const int64_t* x, int64_t ld, int B, int T, int d, int64_t* dst, cudaStream_t st) {
    if (B <= 0) return 0;
    k_gather_last<<<dim3((unsigned)((d + 127) / 128), (unsigned)B), 128, 0, st>>>(x, ld, T, d, dst);
    return 1;
}

int argmax_vocab(const int64_t* last, int B, int d, const WDesc& tok, int vocab, int scale_bits,
                 unsigned long long* keys, int32_t* ids, cudaStream_t st) {
    if (B <= 0) return 0;
    int64_t rows = tok.elements / d;
    if (vocab > rows) vocab = (int)rows;
    cudaMemsetAsync(keys, 0, sizeof(unsigned long long) * B, st);
    if (vocab > 0) {
        const double sc = ldexp(1.0, -scale_bits);
        switch (tok.dtype) {
            case DT_Q4_0: launch_argmax<DT_Q4_0>(last, B, d, tok, vocab, sc, keys, st); break;
            case DT_Q8_0: launch_argmax<DT_Q8_0>(last, B, d, tok, vocab, sc, keys, st); break;
            case DT_F16: launch_argmax<DT_F16>(last, B, d, tok, vocab, sc, keys, st); break;
            case DT_BF16: launch_argmax<DT_BF16>(last, B, d, tok, vocab, sc, keys, st); break;
            default: launch_argmax<DT_F32>(last, B, d, tok, vocab, sc, keys, st); break;
        }
    }
    k_keys_to_ids<<<(B + 127) / 128, 128, 0, st>>>(keys, B, ids);
    return 1 + (vocab > 0 ? 1 : 0);
}

}  // namespace slx
