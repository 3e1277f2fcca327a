// k_vocab.cu -- the VocabLattice lm-head of the causal LM on the device.
//
// Generate(useLattice: true, latticeK) (Gguf/IntegerCausalSource.cs:86-108, PredictNextToken :149-157)
// replaces the full-vocabulary argmax with a k-nearest-neighbour query: VocabLattice
// (Lattice/VocabLattice.cs:15-41) holds every row of TokenEmbeddingsFloat ((float)Half of the token
// table, IntegerCausalSource.cs:51-62) quantized by EmbeddingAdapter.Quantize with ZeroThreshold 0.001
// and GlobalScale 1e9; QueryTopK (:43-58) quantizes the float hidden state the same way and returns the
// k rows nearest by SparseVector.DistanceSquaredL2Fast; ScoreCandidates (:60-76) takes the sequential
// fp32 dot of each candidate row with the hidden state and the highest score wins.
//
// Device form. The table is kept once, as the Half bits of the token rows (2 bytes per component);
// each row's quantized components are recomputed from those bits while the distances stream, which
// reads a quarter of the bytes a stored int64 lattice would. The distance is the reference's wrapping
// sum of (ulong)((a-b)*(a-b)); in arithmetic mod 2^64 it equals sum a^2 + sum b^2 - 2 sum a*b, so each
// (row, query) pair costs one 64-bit multiply-add per component and the two norms are computed once.
// A block-wide radix select keeps the k smallest (distance, row) pairs and a bitonic sort orders them;
// equal distances go in ascending row order (the reference's KnnHeap leaves them to heap order).
// ScoreCandidates' Array.Sort is unstable as well: among equal highest scores the candidate nearest in
// (distance, row) order wins here, and a NaN score loses to every number (float.CompareTo).
#include <cstdint>
#include <string>

#include <cuda_runtime.h>

#include "slx_device.cuh"
#include "slx_kernels.h"
#include "slx_status.h"
#include "slx_vocab.h"

namespace slx {
namespace vocab {
namespace {

constexpr float ZERO_THRESHOLD = 0.001f;
constexpr double GLOBAL_SCALE = 1e9;

// EmbeddingAdapter.Quantize of one component (Math/EmbeddingAdapter.cs:15-41, no sparsity budget):
// |f| < ZeroThreshold -> 0, else (long)(f * (double)GlobalScale). The double product is exact.
SLX_DEV int64_t quantize(float f) { return fabsf(f) < ZERO_THRESHOLD ? 0 : cs_d2l((double)f * GLOBAL_SCALE); }

__global__ void k_vocab_table(WDesc tok, int64_t total, uint16_t* __restrict__ table) {
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x)
        table[e] = f2h(dequant_elem(tok.dtype, tok.data, e, tok.nblocks));
}

// ForwardCausalFloat (IntegerCausalSource.cs:114-122): h = (float)(last * 2^-s), then its quantization.
__global__ void k_vocab_hidden(const int64_t* __restrict__ last, int64_t total, double scale, float* __restrict__ hf,
                               int64_t* __restrict__ hq) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= total) return;
    const float h = __double2float_rn((double)last[i] * scale);
    hf[i] = h;
    hq[i] = quantize(h);
}

__global__ void k_vocab_quantize(const float* __restrict__ hf, int64_t total, int64_t* __restrict__ hq) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i < total) hq[i] = quantize(hf[i]);
}

SLX_DEV uint64_t warp_sum(uint64_t s) {
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, (unsigned long long)s, o);
    return s;
}

// hn[b] = sum_j hq[b][j]^2 mod 2^64, one warp per query.
__global__ void k_vocab_norms(const int64_t* __restrict__ hq, int B, int d, uint64_t* __restrict__ hn) {
    const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (b >= B) return;
    uint64_t s = 0;
    for (int j = lane; j < d; j += 32) {
        const uint64_t x = (uint64_t)hq[(int64_t)b * d + j];
        s += x * x;
    }
    s = warp_sum(s);
    if (lane == 0) hn[b] = s;
}

// dist[q0+i][v] for the g <= DG queries q0.. staged in shared memory: each warp takes two vocabulary
// rows at a time, lanes stride the components (coalesced Half loads, conflict-free int64 shared reads).
constexpr int DG = 8;
constexpr int DWARPS = 8;
constexpr int SMEM_CAP = 200 * 1024;
__global__ void __launch_bounds__(DWARPS * 32) k_vocab_dist(const uint16_t* __restrict__ table, int64_t V, int d,
                                                            const int64_t* __restrict__ hq,
                                                            const uint64_t* __restrict__ hn, int q0, int g,
                                                            uint64_t* __restrict__ dist) {
    extern __shared__ int64_t sh[];  // [g][d]
    for (int64_t i = threadIdx.x; i < (int64_t)g * d; i += blockDim.x) sh[i] = hq[(int64_t)q0 * d + i];
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int64_t v0 = ((int64_t)blockIdx.x * DWARPS + warp) * 2; v0 < V; v0 += (int64_t)gridDim.x * DWARPS * 2) {
        const bool two = v0 + 1 < V;
        const uint16_t* r0 = table + v0 * d;
        const uint16_t* r1 = two ? r0 + d : r0;
        uint64_t na = 0, nb = 0, a[DG], b[DG];
#pragma unroll
        for (int i = 0; i < DG; i++) a[i] = b[i] = 0;
        for (int j = lane; j < d; j += 32) {
            const uint64_t ea = (uint64_t)quantize(h2f(r0[j]));
            const uint64_t eb = (uint64_t)quantize(h2f(r1[j]));
            na += ea * ea;
            nb += eb * eb;
#pragma unroll
            for (int i = 0; i < DG; i++) {
                if (i < g) {
                    const uint64_t h = (uint64_t)sh[i * d + j];
                    a[i] += h * ea;
                    b[i] += h * eb;
                }
            }
        }
        na = warp_sum(na);
        nb = warp_sum(nb);
        uint64_t mine = 0;
#pragma unroll
        for (int i = 0; i < DG; i++) {
            if (i < g) {
                const uint64_t sa = warp_sum(a[i]), sb = warp_sum(b[i]);
                if (lane == i) mine = sa;
                if (lane == 16 + i) mine = sb;
            }
        }
        // lane i writes query q0+i of row v0, lane 16+i of row v0+1
        const int i = lane & 15;
        if (i < g && (lane < 16 || two)) {
            const uint64_t e2 = lane < 16 ? na : nb;
            dist[(int64_t)(q0 + i) * V + v0 + (lane >> 4)] = hn[q0 + i] + e2 - 2 * mine;
        }
    }
}

// The k smallest (distance, row) of dist[b][0..V) in ascending order, one block per query: an MSB-first
// radix select over the eight distance bytes finds the k-th smallest distance D; every row below D is
// gathered, rows equal to D are taken in ascending row order until there are k, and a bitonic sort
// orders the pairs. Requires 1 <= k <= min(V, KMAX).
constexpr int TK = 1024;
__global__ void __launch_bounds__(TK) k_vocab_topk(const uint64_t* __restrict__ dist, int64_t V, int k,
                                                   int32_t* __restrict__ out) {
    extern __shared__ uint64_t key_d[];  // [n2], then int32 key_i[n2]
    __shared__ unsigned int hist[256];
    __shared__ int warp_cnt[TK / 32];
    __shared__ uint64_t s_prefix;
    __shared__ int s_remaining, s_count, s_eq_taken;
    int n2 = 1;
    while (n2 < k) n2 <<= 1;
    int32_t* key_i = (int32_t*)(key_d + n2);
    const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint64_t* row = dist + (int64_t)b * V;
    if (tid == 0) {
        s_prefix = 0;
        s_remaining = k;
        s_count = 0;
        s_eq_taken = 0;
    }
    for (int pass = 7; pass >= 0; pass--) {
        if (tid < 256) hist[tid] = 0;
        __syncthreads();
        const uint64_t prefix = s_prefix;
        const uint64_t hi_mask = pass == 7 ? 0 : ~0ull << (8 * (pass + 1));
        for (int64_t v = tid; v < V; v += TK) {
            const uint64_t x = row[v];
            if ((x & hi_mask) == prefix) atomicAdd(&hist[(x >> (8 * pass)) & 255], 1u);
        }
        __syncthreads();
        if (tid == 0) {
            unsigned int below = 0;
            int bin = 0;
            for (; bin < 255; bin++) {
                if (below + hist[bin] >= (unsigned)s_remaining) break;
                below += hist[bin];
            }
            s_prefix = prefix | ((uint64_t)bin << (8 * pass));
            s_remaining -= (int)below;
        }
        __syncthreads();
    }
    const uint64_t D = s_prefix;  // the k-th smallest distance
    const int need_eq = s_remaining;
    for (int64_t v = tid; v < V; v += TK) {
        const uint64_t x = row[v];
        if (x < D) {
            const int p = atomicAdd(&s_count, 1);
            key_d[p] = x;
            key_i[p] = (int32_t)v;
        }
    }
    __syncthreads();
    const int base = s_count;  // = k - need_eq
    for (int64_t v0 = 0; v0 < V; v0 += TK) {
        if (s_eq_taken >= need_eq) break;  // uniform: read after a barrier
        const int64_t v = v0 + tid;
        const bool f = v < V && row[v] == D;
        const unsigned m = __ballot_sync(0xffffffffu, f);
        if (lane == 0) warp_cnt[warp] = __popc(m);
        __syncthreads();
        int off = s_eq_taken + __popc(m & ((1u << lane) - 1));
        for (int w = 0; w < warp; w++) off += warp_cnt[w];
        if (f && off < need_eq) {
            key_d[base + off] = D;
            key_i[base + off] = (int32_t)v;
        }
        __syncthreads();
        if (tid == 0) {
            int total = 0;
            for (int w = 0; w < TK / 32; w++) total += warp_cnt[w];
            s_eq_taken = min(need_eq, s_eq_taken + total);
        }
        __syncthreads();
    }
    for (int i = k + tid; i < n2; i += TK) {
        key_d[i] = UINT64_MAX;
        key_i[i] = INT32_MAX;
    }
    __syncthreads();
    for (int size = 2; size <= n2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < n2; i += TK) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool up = (i & size) == 0;
                    const bool gt = key_d[i] > key_d[j] || (key_d[i] == key_d[j] && key_i[i] > key_i[j]);
                    if (gt == up) {
                        const uint64_t td = key_d[i];
                        key_d[i] = key_d[j];
                        key_d[j] = td;
                        const int32_t ti = key_i[i];
                        key_i[i] = key_i[j];
                        key_i[j] = ti;
                    }
                }
            }
            __syncthreads();
        }
    }
    for (int i = tid; i < k; i += TK) out[(int64_t)b * k + i] = key_i[i];
}

// ScoreCandidates (Lattice/VocabLattice.cs:60-76) and the first entry of its descending sort, one block
// per query. Each candidate's dot is the reference's sequential fp32 multiply-then-add. The winner is
// the largest key (score order, -0 counted as +0, NaN below every number; then the earlier candidate).
SLX_DEV uint32_t ordered(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
constexpr int ST = 256;
__global__ void __launch_bounds__(ST) k_vocab_score(const uint16_t* __restrict__ table, int d,
                                                    const float* __restrict__ hf, const int32_t* __restrict__ cand,
                                                    int k, int eos, int32_t* __restrict__ next) {
    extern __shared__ float hs[];  // [d]
    __shared__ unsigned long long best;
    const int b = blockIdx.x, tid = threadIdx.x;
    for (int j = tid; j < d; j += ST) hs[j] = hf[(int64_t)b * d + j];
    if (tid == 0) best = 0;
    __syncthreads();
    unsigned long long key = 0;
    for (int c = tid; c < k; c += ST) {
        const uint16_t* row = table + (int64_t)cand[(int64_t)b * k + c] * d;
        float dot = 0.0f;
        for (int j = 0; j < d; j++) dot = __fadd_rn(dot, __fmul_rn(hs[j], h2f(row[j])));
        dot = __fadd_rn(dot, 0.0f);  // -0 -> +0: the two compare equal
        const unsigned long long kc =
            ((unsigned long long)(isnan(dot) ? 0u : ordered(dot)) << 32) | (0xFFFFFFFFu - (uint32_t)c);
        key = kc > key ? kc : key;
    }
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, o);
        key = k2 > key ? k2 : key;
    }
    if ((tid & 31) == 0 && key) atomicMax(&best, key);
    __syncthreads();
    if (tid == 0) next[b] = k > 0 ? cand[(int64_t)b * k + (0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFu))] : eos;
}

bool grow(void** p, size_t& cap, size_t need) {
    if (need == 0) need = 1;
    if (need <= cap) return true;
    if (*p) cudaFree(*p);
    *p = nullptr;
    cap = 0;
    if (cudaMalloc(p, need) != cudaSuccess) return false;
    cap = need;
    return true;
}

int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

int queries_per_pass(int d) {
    int g = SMEM_CAP / (8 * d);
    return g < DG ? g : DG;
}

// Norms, distances and the radix select for the B queries quantized in L.hq; k in [1, V].
int candidates(Lattice& L, int B, int k, cudaStream_t st) {
    int n = 0;
    k_vocab_norms<<<(unsigned)((B + 7) / 8), 256, 0, st>>>(L.hq, B, L.d, L.hn);
    n++;
    const int gmax = queries_per_pass(L.d);
    static int configured = 0;
    const int smem_max = gmax * L.d * 8;
    if (smem_max > 48 * 1024 && smem_max > configured) {
        cudaFuncSetAttribute(k_vocab_dist, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_max);
        configured = smem_max;
    }
    for (int q0 = 0; q0 < B; q0 += gmax) {
        const int g = B - q0 < gmax ? B - q0 : gmax;
        const int smem = g * L.d * 8;
        int per_sm = 1;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_vocab_dist, DWARPS * 32, smem);
        if (per_sm < 1) per_sm = 1;
        const int64_t want = (L.V + DWARPS * 2 - 1) / (DWARPS * 2);
        const int64_t cap = (int64_t)sm_count() * per_sm;
        k_vocab_dist<<<(unsigned)(want < cap ? want : cap), DWARPS * 32, smem, st>>>(L.table, L.V, L.d, L.hq, L.hn, q0,
                                                                                    g, L.dist);
        n++;
    }
    int n2 = 1;
    while (n2 < k) n2 <<= 1;
    const int tsmem = n2 * 12;
    static int tconfigured = 0;
    if (tsmem > 48 * 1024 && tsmem > tconfigured) {
        cudaFuncSetAttribute(k_vocab_topk, cudaFuncAttributeMaxDynamicSharedMemorySize, tsmem);
        tconfigured = tsmem;
    }
    k_vocab_topk<<<(unsigned)B, TK, tsmem, st>>>(L.dist, L.V, k, L.cand);
    return n + 1;
}
}  // namespace

int build(const WDesc& tok, int64_t vocab, int d, Lattice& L, cudaStream_t st, std::string& err) {
    release(L);
    if (d <= 0 || 8 * d > SMEM_CAP) {
        err = "vocab lattice: embedding width must be in [1, 25600]";
        return SLX_EINVAL;
    }
    const int64_t rows = tok.elements / d;
    L.V = vocab < rows ? vocab : rows;
    if (L.V < 0) L.V = 0;
    if (L.V > INT32_MAX) {
        err = "vocab lattice: more rows than int32 token ids";
        return SLX_EINVAL;
    }
    L.d = d;
    const int64_t total = L.V * d;
    if (cudaMalloc(&L.table, sizeof(uint16_t) * (total > 0 ? total : 1)) != cudaSuccess) {
        L.table = nullptr;
        err = "vocab lattice: device allocation failed";
        return SLX_EOOM;
    }
    if (total > 0) k_vocab_table<<<(unsigned)(sm_count() * 8), 256, 0, st>>>(tok, total, L.table);
    if (cudaGetLastError() != cudaSuccess) {
        release(L);
        err = "vocab lattice: table kernel failed to launch";
        return SLX_ECUDA;
    }
    return SLX_OK;
}

void release(Lattice& L) {
    for (void* p : {(void*)L.table, (void*)L.hq, (void*)L.hf, (void*)L.hn, (void*)L.dist, (void*)L.cand})
        if (p) cudaFree(p);
    L = Lattice();
}

int reserve(Lattice& L, int B, int k, std::string& err) {
    const int kc = k > 0 ? k : 1;
    if (!grow((void**)&L.hq, L.hq_bytes, sizeof(int64_t) * (size_t)B * L.d) ||
        !grow((void**)&L.hf, L.hf_bytes, sizeof(float) * (size_t)B * L.d) ||
        !grow((void**)&L.hn, L.hn_bytes, sizeof(uint64_t) * (size_t)B) ||
        !grow((void**)&L.dist, L.dist_bytes, sizeof(uint64_t) * (size_t)B * (size_t)L.V) ||
        !grow((void**)&L.cand, L.cand_bytes, sizeof(int32_t) * (size_t)B * kc)) {
        err = "vocab lattice: device allocation failed";
        return SLX_EOOM;
    }
    return SLX_OK;
}

int query_topk(Lattice& L, int B, int k, int32_t* d_ids, cudaStream_t st) {
    if (B <= 0 || k <= 0) return 0;
    const int keff = (int64_t)k > L.V ? (int)L.V : k;
    const int64_t total = (int64_t)B * L.d;
    int n = 0;
    if (total > 0) {
        k_vocab_quantize<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(L.hf, total, L.hq);
        n++;
    }
    if (keff > 0) {
        n += candidates(L, B, keff, st);
        cudaMemcpy2DAsync(d_ids, sizeof(int32_t) * k, L.cand, sizeof(int32_t) * keff, sizeof(int32_t) * keff, B,
                          cudaMemcpyDeviceToDevice, st);
    }
    if (k > keff)  // past the vocabulary: id -1
        cudaMemset2DAsync((uint8_t*)d_ids + sizeof(int32_t) * keff, sizeof(int32_t) * k, 0xFF,
                          sizeof(int32_t) * (k - keff), B, st);
    return n;
}

int next_tokens(Lattice& L, const int64_t* d_last, int B, int scale_bits, int k, int eos, int32_t* d_next,
                cudaStream_t st) {
    if (B <= 0) return 0;
    const int keff = k <= 0 ? 0 : ((int64_t)k > L.V ? (int)L.V : k);
    const int64_t total = (int64_t)B * L.d;
    int n = 0;
    if (total > 0) {
        k_vocab_hidden<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(d_last, total, ldexp(1.0, -scale_bits), L.hf,
                                                                      L.hq);
        n++;
    }
    if (keff > 0) n += candidates(L, B, keff, st);
    const size_t smem = sizeof(float) * (size_t)L.d;
    static size_t configured = 0;
    if (smem > 48 * 1024 && smem > configured) {
        cudaFuncSetAttribute(k_vocab_score, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        configured = smem;
    }
    k_vocab_score<<<(unsigned)B, ST, smem, st>>>(L.table, L.d, L.hf, L.cand, keff, eos, d_next);
    return n + 1;
}

}  // namespace vocab
}  // namespace slx
