// slx_exact.cuh -- the exact CUDA-core projection GEMM as a device routine, shared by its own
// kernel (k_core.cu: k_gemm_exact) and by the tensor-core GEMM, which runs it in place of its MMAs
// when an activation did not fit its digits (so no separate gated launch follows every projection).
//
// c = (a . w^T) >> shift (+ r): IntegerMatMul.MatMul + DotInt128 (Math/IntegerMatMul.cs:37-76,
// 209-229) with the weight's Q30 composite formed from the packed GGUF blocks. 64 x 64 output
// tiles, K in steps of one 32-element quant block, 4 x 4 Int128 accumulators per thread; the first
// 256 threads of the block compute, every thread of the block takes part in its barriers.
#pragma once
#include "slx_device.cuh"
#include "slx_kernels.h"

namespace slx {

constexpr int XBM = 64, XBN = 64, XBK = 32, XTH = 256;
constexpr size_t XSMEM = 2 * (size_t)XBK * (XBM + 1) * sizeof(int64_t);  // As and Ws

// As, Ws: shared [XBK][XBM + 1] each; tiles tile0, tile0 + tstep, ...
__device__ inline void exact_gemm_tiles(const int64_t* __restrict__ A, int64_t lda, int M, int K, const WDesc& W,
                                        int64_t* __restrict__ C, int64_t ldc, int shift, const int64_t* __restrict__ R,
                                        int64_t ldr, int64_t (*As)[XBM + 1], int64_t (*Ws)[XBN + 1], int tile0,
                                        int tstep) {
    const int tid = threadIdx.x, tx = tid & 15, ty = (tid >> 4) & 15;
    const bool act = tid < XTH;
    const int N = (int)W.N;
    const int ntn = (N + XBN - 1) / XBN, ntiles = ntn * ((M + XBM - 1) / XBM);
    for (int tile = tile0; tile < ntiles; tile += tstep) {
        const int m0 = (tile / ntn) * XBM, n0 = (tile % ntn) * XBN;
        u128 acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[i][j] = 0;
        for (int k0 = 0; k0 < K; k0 += XBK) {
            if (act) {
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int idx = tid + XTH * i, r = idx >> 5, c = idx & 31;
                    const int gm = m0 + r, gk = k0 + c;
                    As[c][r] = (gm < M && gk < K) ? A[(int64_t)gm * lda + gk] : 0;
                }
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int idx = tid + XTH * i, r = idx >> 5, c = idx & 31;
                    const int gn = n0 + r, gk = k0 + c;
                    int64_t w = 0;
                    if (gn < N && gk < K)
                        w = composite(dequant_elem(W.dtype, W.data, (int64_t)gn * K + gk, W.nblocks), W.mode, W.scale);
                    Ws[c][r] = w;
                }
            }
            __syncthreads();
            if (act) {
#pragma unroll 4
                for (int kk = 0; kk < XBK; kk++) {
                    int64_t a[4], w[4];
#pragma unroll
                    for (int i = 0; i < 4; i++) a[i] = As[kk][ty + 16 * i];
#pragma unroll
                    for (int j = 0; j < 4; j++) w[j] = Ws[kk][tx + 16 * j];
#pragma unroll
                    for (int i = 0; i < 4; i++)
#pragma unroll
                        for (int j = 0; j < 4; j++) acc[i][j] += (u128)((i128)a[i] * (i128)w[j]);
                }
            }
            __syncthreads();
        }
        if (act) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int m = m0 + ty + 16 * i;
                if (m >= M) continue;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int n = n0 + tx + 16 * j;
                    if (n >= N) continue;
                    int64_t v = shift > 0 ? lo64(sar128((i128)acc[i][j], shift)) : lo64((i128)acc[i][j]);
                    if (R) v = wadd(v, R[(int64_t)m * ldr + n]);
                    C[(int64_t)m * ldc + n] = v;
                }
            }
        }
        __syncthreads();  // the next tile reuses As / Ws
    }
}

}  // namespace slx
