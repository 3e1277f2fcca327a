// k_float.cu -- TransformerEmbeddingSource, the fp32 twin of the encoder (Gguf/TransformerEmbeddingSource.cs).
//
// The reference reads every weight as float (ReadTensorF32) and runs the encoder graph in fp32:
// BuildEmbeddings, LayerNorm with eps 1e-12, per block QKV -> float RoPE (512-row cache) -> attention
// (scores scaled by 1/sqrt(hd), MathF.Exp softmax, P.V) -> O -> +residual -> LayerNorm -> SiLU-gated
// FFN -> +residual -> LayerNorm, then the mean over all rows and L2 normalisation. Its dot products
// are Vector<float> SIMD sums whose lane order depends on the machine, so this twin is held to a
// tolerance (maximum absolute error and cosine), not to bits.
//
// The projections run on the tensor cores (k_fgemm_tc.cu: operands split into high and low tf32
// parts, three products per pair, fp32 accumulation), which keeps fp32-level precision. The two
// attention contractions, and the projections when the tensor-core path is off, use one fp32 GEMM
// kernel with FFMA accumulation: 128 x 128 output tiles, 8 x 8 per thread, K staged through shared
// memory in steps of 8, arbitrary strides on both operands and a two-level batch (sequence, head).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <vector>

#include <cuda_runtime.h>

#include "slx_float.h"

namespace slx {
namespace fenc {
namespace {

constexpr int TM = 128, TN = 128, TK = 8, GT = 256;

struct GemmF {
    const float* A;
    int64_t a_m, a_k, a_z1, a_z2;  // A(m, k) = A[m*a_m + k*a_k + (z/zdiv)*a_z1 + (z%zdiv)*a_z2]
    const float* B;
    int64_t b_n, b_k, b_z1, b_z2;  // B(n, k)
    float* C;
    int64_t c_m, c_z1, c_z2;       // C(m, n) = C[m*c_m + n + ...]
    int M, N, K, zdiv;
    float alpha;
};

// C = alpha * A . B^T over each batch entry z = blockIdx.z.
__global__ void __launch_bounds__(GT, 2) k_sgemm(GemmF p) {
    __shared__ __align__(16) float As[TK][TM + 4];
    __shared__ __align__(16) float Bs[TK][TN + 4];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN, z = blockIdx.z;
    const float* A = p.A + (int64_t)(z / p.zdiv) * p.a_z1 + (int64_t)(z % p.zdiv) * p.a_z2;
    const float* B = p.B + (int64_t)(z / p.zdiv) * p.b_z1 + (int64_t)(z % p.zdiv) * p.b_z2;
    float* C = p.C + (int64_t)(z / p.zdiv) * p.c_z1 + (int64_t)(z % p.zdiv) * p.c_z2;
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.0f;
    const bool a_kc = p.a_k == 1, b_kc = p.b_k == 1;
    for (int k0 = 0; k0 < p.K; k0 += TK) {
        // 1024 elements of each tile, four per thread; the mapping follows the contiguous index
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int e = tid * 4 + u;
            int mm, kk;
            if (a_kc) { mm = e >> 3; kk = e & 7; } else { kk = e >> 7; mm = e & 127; }
            const int gm = m0 + mm, gk = k0 + kk;
            As[kk][mm] = (gm < p.M && gk < p.K) ? A[(int64_t)gm * p.a_m + (int64_t)gk * p.a_k] : 0.0f;
            int nn, kb;
            if (b_kc) { nn = e >> 3; kb = e & 7; } else { kb = e >> 7; nn = e & 127; }
            const int gn = n0 + nn, gk2 = k0 + kb;
            Bs[kb][nn] = (gn < p.N && gk2 < p.K) ? B[(int64_t)gn * p.b_n + (int64_t)gk2 * p.b_k] : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < TK; kk++) {
            const float4 a0 = *reinterpret_cast<const float4*>(&As[kk][ty * 8]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[kk][ty * 8 + 4]);
            const float4 b0 = *reinterpret_cast<const float4*>(&Bs[kk][tx * 8]);
            const float4 b1 = *reinterpret_cast<const float4*>(&Bs[kk][tx * 8 + 4]);
            const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int gm = m0 + ty * 8 + i;
        if (gm >= p.M) continue;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int gn = n0 + tx * 8 + j;
            if (gn < p.N) C[(int64_t)gm * p.c_m + gn] = p.alpha * acc[i][j];
        }
    }
}

void sgemm(const GemmF& p, int batch, cudaStream_t st) {
    dim3 grid((unsigned)((p.N + TN - 1) / TN), (unsigned)((p.M + TM - 1) / TM), (unsigned)batch);
    k_sgemm<<<grid, GT, 0, st>>>(p);
}

// c[rows][nout] = a[rows][nin] . w[nout][nin]^T (GGUF weights are [out][in] row-major)
void project_ffma(const float* a, int rows, int nin, const float* w, int nout, float* c, cudaStream_t st) {
    GemmF p{};
    p.A = a; p.a_m = nin; p.a_k = 1;
    p.B = w; p.b_n = nin; p.b_k = 1;
    p.C = c; p.c_m = nout;
    p.M = rows; p.N = nout; p.K = nin; p.zdiv = 1; p.alpha = 1.0f;
    sgemm(p, 1, st);
}

// The same product on the tensor cores when the weight's split planes exist (the FFMA kernel
// otherwise, or when the tensor maps cannot be encoded).
void project(const float* a, int rows, int nin, const float* w, const float* w_t, int nout, float* c, Workspace& ws,
             cudaStream_t st) {
    if (w_t && ws.planes && tc_project(a, rows, nin, w_t, nout, c, ws.planes, ws.err, st)) return;
    project_ffma(a, rows, nin, w, nout, c, st);
}

__global__ void k_embed(const int32_t* __restrict__ ids, int64_t total, int d, const float* __restrict__ tok,
                        int64_t tok_rows, const float* __restrict__ tt, int unk, float* __restrict__ x) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= total) return;
    const int64_t r = i / d;
    const int j = (int)(i - r * d);
    int64_t id = ids[r];
    if (id < 0 || id >= tok_rows) id = unk;
    x[i] = tok[id * d + j] + tt[j];
}

// LayerNorm of one row per warp: mean, variance about it, (x - mean) * (1 / sqrt(var + 1e-12)) * w + b.
__global__ void k_layernorm(float* __restrict__ x, int rows, int d, const float* __restrict__ w,
                            const float* __restrict__ b) {
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= rows) return;
    float* row = x + (int64_t)r * d;
    float s = 0.0f;
    for (int j = lane; j < d; j += 32) s += row[j];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / d;
    float v = 0.0f;
    for (int j = lane; j < d; j += 32) {
        const float dl = row[j] - mean;
        v += dl * dl;
    }
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const float inv = 1.0f / sqrtf(v / d + 1e-12f);
    for (int j = lane; j < d; j += 32) row[j] = (row[j] - mean) * inv * w[j] + b[j];
}

// NeoX rotation of the q and k parts of each [q | k | v] row (positions t = row % T).
__global__ void k_rope(float* __restrict__ qkv, int64_t rows, int T, int d, int H, int hd,
                       const float* __restrict__ cs, const float* __restrict__ sn) {
    const int half = hd / 2;
    const int64_t total = rows * 2 * H * half;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int ii = (int)(i % half);
        const int64_t rest = i / half;
        const int h = (int)(rest % H);
        const int part = (int)((rest / H) % 2);
        const int64_t r = rest / (2 * H);
        const int t = (int)(r % T);
        float* p = qkv + r * 3 * d + part * d + h * hd;
        const float c = cs[(int64_t)t * half + ii], s = sn[(int64_t)t * half + ii];
        const float x0 = p[ii], x1 = p[ii + half];
        p[ii] = x0 * c - x1 * s;
        p[ii + half] = x0 * s + x1 * c;
    }
}

// Row softmax in place (warp per row): exp(x - max), then times 1 / sum.
__global__ void k_softmax(float* __restrict__ s, int64_t rows, int n) {
    const int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    float* row = s + r * n;
    float mx = -INFINITY;
    for (int j = lane; j < n; j += 32) mx = fmaxf(mx, row[j]);
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
    for (int j = lane; j < n; j += 32) {
        const float e = expf(row[j] - mx);
        row[j] = e;
        sum += e;
    }
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float inv = 1.0f / sum;
    for (int j = lane; j < n; j += 32) row[j] *= inv;
}

__global__ void k_silu_mul(float* __restrict__ up, const float* __restrict__ gate, int64_t n) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i < n) {
        const float g = gate[i];
        up[i] *= g / (1.0f + expf(-g));
    }
}

__global__ void k_add(float* __restrict__ dst, const float* __restrict__ src, int64_t n) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i < n) dst[i] += src[i];
}

// Mean over the T rows of each sequence, then L2 normalisation (unchanged below 1e-10), one block each.
__global__ void k_pool_l2(const float* __restrict__ x, int T, int d, float* __restrict__ out) {
    extern __shared__ float pooled[];
    __shared__ float part[32];
    const int b = blockIdx.x;
    const float inv = 1.0f / T;
    float sq = 0.0f;
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
        float s = 0.0f;
        for (int t = 0; t < T; t++) s += x[((int64_t)b * T + t) * d + j];
        s *= inv;
        pooled[j] = s;
        sq += s * s;
    }
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sq;
    __syncthreads();
    float norm2 = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) norm2 += part[w];
    const float norm = sqrtf(norm2);
    const float s = norm < 1e-10f ? 1.0f : 1.0f / norm;
    for (int j = threadIdx.x; j < d; j += blockDim.x) out[(int64_t)b * d + j] = norm < 1e-10f ? pooled[j] : pooled[j] * s;
}

unsigned blocks(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }

template <class T>
bool grow(T*& p, size_t& cap, size_t count) {
    if (count <= cap) return true;
    cudaFree(p);
    p = nullptr;
    cap = 0;
    if (cudaMalloc(&p, count * sizeof(T)) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    cap = count;
    return true;
}
}  // namespace

void Workspace::release() {
    for (float* p : {x, qkv, att, h, up, gate, sc, planes}) cudaFree(p);
    int* e = err;
    *this = Workspace();
    err = e;
}

int forward(const Model& m, const int32_t* d_ids, int B, int T, float* d_out, Workspace& ws, cudaStream_t st,
            int64_t* launches) {
    const int d = m.d, H = m.heads, hd = d / H, F = m.ff;
    const int64_t M = (int64_t)B * T;
    if (!grow(ws.x, ws.cx, M * d) || !grow(ws.qkv, ws.cqkv, M * 3 * d) || !grow(ws.att, ws.catt, M * d) ||
        !grow(ws.h, ws.ch, M * d) || !grow(ws.up, ws.cup, M * F) || !grow(ws.gate, ws.cgate, M * F) ||
        !grow(ws.sc, ws.csc, (size_t)B * H * T * T))
        return -1;
    const bool tc = !m.layers.empty() && m.layers[0].qkv_t;
    if (tc && !grow(ws.planes, ws.cplanes, tc_act_bytes((int)M, std::max(d, F)) / sizeof(float))) return -1;
    int64_t nl = 0;
    k_embed<<<blocks(M * d, 256), 256, 0, st>>>(d_ids, M * d, d, m.tok, m.tok_rows, m.tt, m.unk, ws.x);
    k_layernorm<<<blocks(M, 8), 256, 0, st>>>(ws.x, (int)M, d, m.enw, m.enb);
    nl += 2;
    const float scale = 1.0f / sqrtf((float)hd);
    for (const Layer& L : m.layers) {
        project(ws.x, (int)M, d, L.qkv, L.qkv_t, 3 * d, ws.qkv, ws, st);
        k_rope<<<(unsigned)std::min<int64_t>(blocks(M * d, 256), 148 * 32), 256, 0, st>>>(ws.qkv, M, T, d, H, hd, m.cos,
                                                                                          m.sin);
        // scores[b][h][t][s] = scale * q_t . k_s
        GemmF s{};
        s.A = ws.qkv; s.a_m = 3 * d; s.a_k = 1; s.a_z1 = (int64_t)T * 3 * d; s.a_z2 = hd;
        s.B = ws.qkv + d; s.b_n = 3 * d; s.b_k = 1; s.b_z1 = (int64_t)T * 3 * d; s.b_z2 = hd;
        s.C = ws.sc; s.c_m = T; s.c_z1 = (int64_t)H * T * T; s.c_z2 = (int64_t)T * T;
        s.M = T; s.N = T; s.K = hd; s.zdiv = H; s.alpha = scale;
        sgemm(s, B * H, st);
        k_softmax<<<blocks((int64_t)B * H * T, 8), 256, 0, st>>>(ws.sc, (int64_t)B * H * T, T);
        // att[b][t][h*hd + j] = sum_s p[t][s] v_s[j]
        GemmF pv{};
        pv.A = ws.sc; pv.a_m = T; pv.a_k = 1; pv.a_z1 = (int64_t)H * T * T; pv.a_z2 = (int64_t)T * T;
        pv.B = ws.qkv + 2 * d; pv.b_n = 1; pv.b_k = 3 * d; pv.b_z1 = (int64_t)T * 3 * d; pv.b_z2 = hd;
        pv.C = ws.att; pv.c_m = d; pv.c_z1 = (int64_t)T * d; pv.c_z2 = hd;
        pv.M = T; pv.N = hd; pv.K = T; pv.zdiv = H; pv.alpha = 1.0f;
        sgemm(pv, B * H, st);
        project(ws.att, (int)M, d, L.o, L.o_t, d, ws.h, ws, st);
        k_add<<<blocks(M * d, 256), 256, 0, st>>>(ws.h, ws.x, M * d);
        k_layernorm<<<blocks(M, 8), 256, 0, st>>>(ws.h, (int)M, d, L.anw, L.anb);
        project(ws.h, (int)M, d, L.up, L.up_t, F, ws.up, ws, st);
        project(ws.h, (int)M, d, L.gate, L.gate_t, F, ws.gate, ws, st);
        k_silu_mul<<<blocks(M * F, 256), 256, 0, st>>>(ws.up, ws.gate, M * F);
        project(ws.up, (int)M, F, L.down, L.down_t, d, ws.x, ws, st);
        k_add<<<blocks(M * d, 256), 256, 0, st>>>(ws.x, ws.h, M * d);
        k_layernorm<<<blocks(M, 8), 256, 0, st>>>(ws.x, (int)M, d, L.lnw, L.lnb);
        nl += tc ? 19 : 14;
    }
    k_pool_l2<<<(unsigned)B, 256, sizeof(float) * d, st>>>(ws.x, T, d, d_out);
    nl++;
    if (launches) *launches += nl;
    return (int)nl;
}

}  // namespace fenc
}  // namespace slx
