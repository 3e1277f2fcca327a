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

#include "slx_attr.h"
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

// The same for a Half component, in integer arithmetic. A finite Half of magnitude >= 2^-14 is
// M * 2^(E-25) (M = 1024 + fraction, E the exponent field), so f * 1e9 = M * 1953125 * 2^(E-16)
// exactly (1e9 = 1953125 * 2^9), and (long) truncates the magnitude: a shift of M * 1953125 (< 2^32).
// 0x1419 is the smallest Half magnitude that is not below 0.001f; inf and NaN give long.MinValue
// as (long) of a non-finite double does.
constexpr uint32_t HALF_MAG_ZERO_BELOW = 0x1419u;
SLX_DEV int64_t quantize_half(uint32_t bits) {
    const uint32_t mag = bits & 0x7fffu;
    if (mag < HALF_MAG_ZERO_BELOW) return 0;
    if (mag >= 0x7c00u) return INT64_MIN;
    const uint32_t e = mag >> 10;
    const uint64_t p = (uint64_t)(1024u | (mag & 1023u)) * 1953125u;
    const int64_t q = (int64_t)(e >= 16 ? p << (e - 16) : p >> (16 - e));
    return (bits & 0x8000u) ? -q : q;
}

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

// en[v] = sum_j q[v][j]^2 mod 2^64 of the quantized table rows, one warp per row (built once).
__global__ void k_vocab_rownorms(const uint16_t* __restrict__ table, int64_t V, int d, uint64_t* __restrict__ en) {
    const int lane = threadIdx.x & 31;
    for (int64_t v = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); v < V;
         v += (int64_t)gridDim.x * (blockDim.x >> 5)) {
        uint64_t s = 0;
        for (int j = lane; j < d; j += 32) {
            const uint64_t e = (uint64_t)quantize_half(table[v * d + j]);
            s += e * e;
        }
        s = warp_sum(s);
        if (lane == 0) en[v] = s;
    }
}

// dist[q0+i][v] for G queries q0.. staged in shared memory (slots past the g real queries are zero
// and their sums are dropped): each warp takes two vocabulary rows at a time. With d a multiple of 8
// (VEC) every lane loads eight Half components of each row per step (16-byte loads) and the queries
// are staged component-group-major, sh[i][t][j / 8] for component j = 8 (j / 8) + t, so the lanes'
// int64 reads stay contiguous; otherwise lanes stride single components.
constexpr int DG = 8;
constexpr int DWARPS = 16;
constexpr int SMEM_CAP = 200 * 1024;
template <bool VEC, int G>
__global__ void __launch_bounds__(DWARPS * 32) k_vocab_dist(const uint16_t* __restrict__ table, int64_t V, int d,
                                                            const uint64_t* __restrict__ en,
                                                            const int64_t* __restrict__ hq,
                                                            const uint64_t* __restrict__ hn, int q0, int g,
                                                            uint64_t* __restrict__ dist) {
    extern __shared__ int64_t sh[];  // [G][d]
    const int d8 = d >> 3;
    for (int64_t idx = threadIdx.x; idx < (int64_t)G * d; idx += blockDim.x) {
        const int64_t i = idx / d;
        const int j = (int)(idx - i * d);
        sh[VEC ? i * d + (int64_t)(j & 7) * d8 + (j >> 3) : idx] = i < g ? hq[(int64_t)q0 * d + idx] : 0;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int64_t v0 = ((int64_t)blockIdx.x * DWARPS + warp) * 2; v0 < V; v0 += (int64_t)gridDim.x * DWARPS * 2) {
        const bool two = v0 + 1 < V;
        const uint16_t* r0 = table + v0 * d;
        const uint16_t* r1 = two ? r0 + d : r0;
        uint64_t a[G], b[G];
#pragma unroll
        for (int i = 0; i < G; i++) a[i] = b[i] = 0;
        if constexpr (VEC) {
            const uint4* R0 = reinterpret_cast<const uint4*>(r0);
            const uint4* R1 = reinterpret_cast<const uint4*>(r1);
#pragma unroll 1
            for (int cb = lane; cb < d8; cb += 32) {
                const uint4 x0 = __ldg(R0 + cb), x1 = __ldg(R1 + cb);
                const uint32_t w0[4] = {x0.x, x0.y, x0.z, x0.w}, w1[4] = {x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                for (int t = 0; t < 8; t++) {
                    const uint64_t ea = (uint64_t)quantize_half((w0[t >> 1] >> (16 * (t & 1))) & 0xFFFFu);
                    const uint64_t eb = (uint64_t)quantize_half((w1[t >> 1] >> (16 * (t & 1))) & 0xFFFFu);
#pragma unroll
                    for (int i = 0; i < G; i++) {
                        const uint64_t h = (uint64_t)sh[(int64_t)i * d + t * d8 + cb];
                        a[i] += h * ea;
                        b[i] += h * eb;
                    }
                }
            }
        } else {
            for (int j = lane; j < d; j += 32) {
                const uint64_t ea = (uint64_t)quantize_half(r0[j]);
                const uint64_t eb = (uint64_t)quantize_half(r1[j]);
#pragma unroll
                for (int i = 0; i < G; i++) {
                    const uint64_t h = (uint64_t)sh[i * d + j];
                    a[i] += h * ea;
                    b[i] += h * eb;
                }
            }
        }
        uint64_t mine = 0;
#pragma unroll
        for (int i = 0; i < G; i++) {
            const uint64_t sa = warp_sum(a[i]), sb = warp_sum(b[i]);
            if (lane == i) mine = sa;
            if (lane == 16 + i) mine = sb;
        }
        // lane i writes query q0+i of row v0, lane 16+i of row v0+1
        const int i = lane & 15;
        if (i < g && (lane < 16 || two)) {
            const int64_t v = v0 + (lane >> 4);
            dist[(int64_t)(q0 + i) * V + v] = hn[q0 + i] + en[v] - 2 * mine;
        }
    }
}

// ---- top-k selection --------------------------------------------------------------------------
// The k smallest (distance, row) pairs of a query, ties by ascending row: a radix select finds the
// k-th smallest distance D, every row below D is kept, and rows equal to D are kept in ascending row
// order until there are k. The select starts at the highest byte in which the candidates' minimum and
// maximum differ (the bytes above are common to all of them) and each warp adds its lanes' equal bins
// once (__match_any_sync), since distances crowd into few bins.
//
// Stage 1 (k_topk_slice, k <= SLICE / 4): one block per (slice of SLICE rows, query) holds the slice's
// distances in shared memory, selects its min(k, rows) smallest and writes them in ascending row
// order, padding its KK = min(k, SLICE) slots with (UINT64_MAX, -) marked by id INT32_MAX. Stage 2
// (k_topk_merge) selects the k smallest of those candidates (or of all rows when k is large) and sorts
// them; its candidates are already in ascending row order, so equal distances are taken by row.
constexpr int SLICE = 2048, ST1 = 256;
constexpr int TK = 1024;
constexpr int32_t NO_ROW = INT32_MAX;

// Exclusive prefix sum over the block's threads (warp_sums holds one int per warp); returns the
// exclusive prefix and stores the block total in *total.
template <int NT>
SLX_DEV int block_exclusive_scan(int v, int* warp_sums, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    int before = 0, all = 0;
    for (int w = 0; w < NT / 32; w++) {
        const int c = warp_sums[w];
        before += w < warp ? c : 0;
        all += c;
    }
    __syncthreads();
    *total = all;
    return before + x - v;
}

// Radix select over n values (shared or global, generic addressing) with a validity predicate:
// returns D (the k-th smallest valid value) and *need_eq (how many values equal to D belong to the k).
template <int NT, class Get>
SLX_DEV uint64_t radix_select(int64_t n, int k, Get get, unsigned* hist, uint64_t* wmin, uint64_t* wmax,
                              uint64_t* s_prefix, int* s_remaining, int* s_top, int* need_eq) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint64_t mn = UINT64_MAX, mx = 0;
    for (int64_t i = tid; i < n; i += NT) {
        bool ok;
        const uint64_t x = get(i, ok);
        if (ok) {
            mn = x < mn ? x : mn;
            mx = x > mx ? x : mx;
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const uint64_t a = __shfl_xor_sync(0xffffffffu, (unsigned long long)mn, o);
        const uint64_t c = __shfl_xor_sync(0xffffffffu, (unsigned long long)mx, o);
        mn = a < mn ? a : mn;
        mx = c > mx ? c : mx;
    }
    if (lane == 0) {
        wmin[warp] = mn;
        wmax[warp] = mx;
    }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < NT / 32; w++) {
            mn = wmin[w] < mn ? wmin[w] : mn;
            mx = wmax[w] > mx ? wmax[w] : mx;
        }
        const uint64_t diff = mn ^ mx;
        *s_top = diff ? (63 - __clzll((long long)diff)) >> 3 : -1;
        *s_prefix = *s_top < 0 ? mn : (*s_top == 7 ? 0 : mn & (~0ull << (8 * (*s_top + 1))));
        *s_remaining = k;
    }
    __syncthreads();
    for (int pass = *s_top; pass >= 0; pass--) {
        if (tid < 256) hist[tid] = 0;
        __syncthreads();
        const uint64_t prefix = *s_prefix;
        const uint64_t hi_mask = pass == 7 ? 0 : ~0ull << (8 * (pass + 1));
        for (int64_t i0 = 0; i0 < n; i0 += NT) {
            const int64_t i = i0 + tid;
            unsigned bin = 256;
            if (i < n) {
                bool ok;
                const uint64_t x = get(i, ok);
                if (ok && (x & hi_mask) == prefix) bin = (unsigned)(x >> (8 * pass)) & 255u;
            }
            const unsigned same = __match_any_sync(0xffffffffu, bin);
            if (bin < 256 && lane == __ffs(same) - 1) atomicAdd(&hist[bin], (unsigned)__popc(same));
        }
        __syncthreads();
        if (tid == 0) {
            unsigned int below = 0;
            int bin = 0;
            for (; bin < 255; bin++) {
                if (below + hist[bin] >= (unsigned)*s_remaining) break;
                below += hist[bin];
            }
            *s_prefix = prefix | ((uint64_t)bin << (8 * pass));
            *s_remaining -= (int)below;
        }
        __syncthreads();
    }
    *need_eq = *s_remaining;
    return *s_prefix;
}

__global__ void __launch_bounds__(ST1) k_topk_slice(const uint64_t* __restrict__ dist, int64_t V, int k, int G, int KK,
                                                    uint64_t* __restrict__ cd, int32_t* __restrict__ ci) {
    __shared__ uint64_t xs[SLICE];
    __shared__ unsigned hist[256];
    __shared__ uint64_t wmin[ST1 / 32], wmax[ST1 / 32], s_prefix;
    __shared__ int wsum[ST1 / 32], s_remaining, s_top;
    const int s = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const int64_t r0 = (int64_t)s * SLICE;
    const int n = (int)(V - r0 < SLICE ? V - r0 : SLICE);
    const int kk = k < n ? k : n;
    const uint64_t* row = dist + (int64_t)b * V + r0;
    for (int i = tid; i < SLICE; i += ST1) xs[i] = i < n ? row[i] : UINT64_MAX;
    __syncthreads();
    int need_eq;
    const uint64_t D = radix_select<ST1>(
        n, kk, [&](int64_t i, bool& ok) { ok = true; return xs[i]; }, hist, wmin, wmax, &s_prefix, &s_remaining, &s_top,
        &need_eq);
    // thread t owns rows 8t .. 8t+7 of the slice: both scans keep row order
    constexpr int PER = SLICE / ST1;
    int eqc = 0;
#pragma unroll
    for (int u = 0; u < PER; u++) {
        const int i = tid * PER + u;
        eqc += (i < n && xs[i] == D) ? 1 : 0;
    }
    int tot;
    int eq_rank = block_exclusive_scan<ST1>(eqc, wsum, &tot);
    bool sel[PER];
    int selc = 0;
#pragma unroll
    for (int u = 0; u < PER; u++) {
        const int i = tid * PER + u;
        const uint64_t x = xs[i];
        bool t = false;
        if (i < n) {
            if (x < D) t = true;
            else if (x == D) t = eq_rank++ < need_eq;
        }
        sel[u] = t;
        selc += t;
    }
    int pos = block_exclusive_scan<ST1>(selc, wsum, &tot);
    uint64_t* od = cd + ((int64_t)b * G + s) * KK;
    int32_t* oi = ci + ((int64_t)b * G + s) * KK;
#pragma unroll
    for (int u = 0; u < PER; u++) {
        if (sel[u]) {
            const int i = tid * PER + u;
            od[pos] = xs[i];
            oi[pos] = (int32_t)(r0 + i);
            pos++;
        }
    }
    for (int p = kk + tid; p < KK; p += ST1) {
        od[p] = UINT64_MAX;
        oi[p] = NO_ROW;
    }
}

// Stage 2: the k smallest of n candidates per query (vals[b][0..n), ids[b][0..n) or the index when
// ids is null; id NO_ROW marks an empty slot), sorted by (distance, row). The candidates are staged
// in shared memory when they fit. Requires 1 <= k <= valid candidates, k <= KMAX.
__global__ void __launch_bounds__(TK) k_topk_merge(const uint64_t* __restrict__ vals, const int32_t* __restrict__ ids,
                                                   int64_t n, int k, int staged, int32_t* __restrict__ out,
                                                   uint64_t* __restrict__ out_d) {
    extern __shared__ uint64_t dyn[];  // key_d[n2], key_i[n2], then (staged) sv[n], si[n]
    __shared__ unsigned hist[256];
    __shared__ int warp_cnt[TK / 32];
    __shared__ uint64_t wmin[TK / 32], wmax[TK / 32], s_prefix;
    __shared__ int s_remaining, s_count, s_eq_taken, s_top;
    int n2 = 1;
    while (n2 < k) n2 <<= 1;
    uint64_t* key_d = dyn;
    int32_t* key_i = (int32_t*)(key_d + n2);
    const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint64_t* row = vals + (int64_t)b * n;
    const int32_t* irow = ids ? ids + (int64_t)b * n : nullptr;
    if (staged) {
        uint64_t* sv = (uint64_t*)(key_i + n2 + (n2 & 1));  // 8-byte aligned after key_i
        int32_t* si = (int32_t*)(sv + n);
        for (int64_t i = tid; i < n; i += TK) {
            sv[i] = row[i];
            si[i] = irow ? irow[i] : (int32_t)i;
        }
        row = sv;
        irow = si;
        __syncthreads();
    }
    if (tid == 0) {
        s_count = 0;
        s_eq_taken = 0;
    }
    auto get = [&](int64_t i, bool& ok) {
        ok = !irow || irow[i] != NO_ROW;
        return row[i];
    };
    int need_eq;
    const uint64_t D = radix_select<TK>(n, k, get, hist, wmin, wmax, &s_prefix, &s_remaining, &s_top, &need_eq);
    for (int64_t i = tid; i < n; i += TK) {
        bool ok;
        const uint64_t x = get(i, ok);
        if (ok && x < D) {
            const int p = atomicAdd(&s_count, 1);
            key_d[p] = x;
            key_i[p] = irow ? irow[i] : (int32_t)i;
        }
    }
    __syncthreads();
    const int base = s_count;  // = k - need_eq
    for (int64_t i0 = 0; i0 < n; i0 += TK) {
        if (s_eq_taken >= need_eq) break;  // uniform: read after a barrier
        const int64_t i = i0 + tid;
        bool f = false;
        if (i < n) {
            bool ok;
            const uint64_t x = get(i, ok);
            f = ok && x == D;
        }
        const unsigned m = __ballot_sync(0xffffffffu, f);
        if (lane == 0) warp_cnt[warp] = __popc(m);
        __syncthreads();
        int off = s_eq_taken + __popc(m & ((1u << lane) - 1));
        for (int w = 0; w < warp; w++) off += warp_cnt[w];
        if (f && off < need_eq) {
            key_d[base + off] = D;
            key_i[base + off] = irow ? irow[i] : (int32_t)i;
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
    for (int i = tid; i < k; i += TK) {
        out[(int64_t)b * k + i] = key_i[i];
        if (out_d) out_d[(int64_t)b * k + i] = key_d[i];
    }
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
        if ((d & 7) == 0) {  // 16-byte row loads, issued ahead of the sequential chain
            const uint4* R = reinterpret_cast<const uint4*>(row);
#pragma unroll 4
            for (int cb = 0; cb < (d >> 3); cb++) {
                const uint4 x = __ldg(R + cb);
                const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
                for (int t = 0; t < 8; t++)
                    dot = __fadd_rn(dot, __fmul_rn(hs[cb * 8 + t], h2f((uint16_t)(w[t >> 1] >> (16 * (t & 1))))));
            }
        } else {
            for (int j = 0; j < d; j++) dot = __fadd_rn(dot, __fmul_rn(hs[j], h2f(row[j])));
        }
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

int sm_count() { return slx::device_sm_count(); }

// Stage-1 candidate slots per query: KK = k per slice of SLICE rows.
size_t slice_slots(int64_t V, int k) {
    if (k <= 0 || k > SLICE / 4 || V <= SLICE) return 1;
    return (size_t)((V + SLICE - 1) / SLICE) * (size_t)k;
}

// Queries per distance pass: a power of two (the kernel's template slots) whose int64 rows fit SMEM_CAP.
int queries_per_pass(int d) {
    int g = DG;
    while (g > 1 && g * 8 * d > SMEM_CAP) g >>= 1;
    return g;
}

template <bool VEC, int G>
void launch_dist_t(Lattice& L, int q0, int g, cudaStream_t st) {
    const int smem = G * L.d * 8;
    slx::ensure_smem((const void*)k_vocab_dist<VEC, G>, (size_t)smem);
    int per_sm = 1;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_vocab_dist<VEC, G>, DWARPS * 32, smem);
    if (per_sm < 1) per_sm = 1;
    const int64_t want = (L.V + DWARPS * 2 - 1) / (DWARPS * 2);
    const int64_t cap = (int64_t)sm_count() * per_sm;
    k_vocab_dist<VEC, G><<<(unsigned)(want < cap ? want : cap), DWARPS * 32, smem, st>>>(L.table, L.V, L.d, L.en, L.hq,
                                                                                      L.hn, q0, g, L.dist);
}

void launch_dist(Lattice& L, bool vec, int G, int q0, int g, cudaStream_t st) {
    if (vec) {
        if (G == 1) launch_dist_t<true, 1>(L, q0, g, st);
        else if (G == 2) launch_dist_t<true, 2>(L, q0, g, st);
        else if (G == 4) launch_dist_t<true, 4>(L, q0, g, st);
        else launch_dist_t<true, 8>(L, q0, g, st);
    } else {
        if (G == 1) launch_dist_t<false, 1>(L, q0, g, st);
        else if (G == 2) launch_dist_t<false, 2>(L, q0, g, st);
        else if (G == 4) launch_dist_t<false, 4>(L, q0, g, st);
        else launch_dist_t<false, 8>(L, q0, g, st);
    }
}

// Norms, distances and the radix select for the B queries quantized in L.hq; k in [1, V].
int candidates(Lattice& L, int B, int k, bool want_dist, cudaStream_t st) {
    int n = 0;
    k_vocab_norms<<<(unsigned)((B + 7) / 8), 256, 0, st>>>(L.hq, B, L.d, L.hn);
    n++;
    const int gmax = queries_per_pass(L.d);
    for (int q0 = 0; q0 < B; q0 += gmax) {
        const int g = B - q0 < gmax ? B - q0 : gmax;
        const int G = g <= 1 ? 1 : g <= 2 ? 2 : g <= 4 ? 4 : 8;
        launch_dist(L, (L.d & 7) == 0, G, q0, g, st);
        n++;
    }
    int n2 = 1;
    while (n2 < k) n2 <<= 1;
    const uint64_t* vals = L.dist;
    const int32_t* ids = nullptr;
    int64_t n_cand = L.V;
    if (k <= SLICE / 4 && L.V > SLICE) {
        const int G = (int)((L.V + SLICE - 1) / SLICE), KK = k;
        k_topk_slice<<<dim3((unsigned)G, (unsigned)B), ST1, 0, st>>>(L.dist, L.V, k, G, KK, L.sel_d, L.sel_i);
        n++;
        vals = L.sel_d;
        ids = L.sel_i;
        n_cand = (int64_t)G * KK;
    }
    const size_t keys = (size_t)n2 * 12 + 8;
    const size_t stage = (size_t)n_cand * 12;
    const int staged = keys + stage <= 160 * 1024 ? 1 : 0;
    const int tsmem = (int)(keys + (staged ? stage : 0));
    // the largest request is 160 KiB (staged); unstaged <= KMAX * 12 + 8
    if (tsmem > 48 * 1024) slx::ensure_smem((const void*)k_topk_merge, 160 * 1024);
    k_topk_merge<<<(unsigned)B, TK, tsmem, st>>>(vals, ids, n_cand, k, staged, L.cand, want_dist ? L.cdist : nullptr);
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
    if (cudaMalloc(&L.en, sizeof(uint64_t) * (L.V > 0 ? L.V : 1)) != cudaSuccess) {
        L.en = nullptr;
        release(L);
        err = "vocab lattice: device allocation failed";
        return SLX_EOOM;
    }
    if (total > 0) {
        k_vocab_table<<<(unsigned)(sm_count() * 8), 256, 0, st>>>(tok, total, L.table);
        k_vocab_rownorms<<<(unsigned)(sm_count() * 4), 256, 0, st>>>(L.table, L.V, d, L.en);
    }
    if (cudaGetLastError() != cudaSuccess) {
        release(L);
        err = "vocab lattice: table kernel failed to launch";
        return SLX_ECUDA;
    }
    return SLX_OK;
}

void release(Lattice& L) {
    for (void* p : {(void*)L.table, (void*)L.en, (void*)L.hq, (void*)L.hf, (void*)L.hn, (void*)L.dist, (void*)L.cand, (void*)L.cdist,
                    (void*)L.sel_d, (void*)L.sel_i})
        if (p) cudaFree(p);
    L = Lattice();
}

int reserve(Lattice& L, int B, int k, std::string& err) {
    const int kc = k > 0 ? k : 1;
    if (!grow((void**)&L.hq, L.hq_bytes, sizeof(int64_t) * (size_t)B * L.d) ||
        !grow((void**)&L.hf, L.hf_bytes, sizeof(float) * (size_t)B * L.d) ||
        !grow((void**)&L.hn, L.hn_bytes, sizeof(uint64_t) * (size_t)B) ||
        !grow((void**)&L.dist, L.dist_bytes, sizeof(uint64_t) * (size_t)B * (size_t)L.V) ||
        !grow((void**)&L.cand, L.cand_bytes, sizeof(int32_t) * (size_t)B * kc) ||
        !grow((void**)&L.cdist, L.cdist_bytes, sizeof(uint64_t) * (size_t)B * kc) ||
        !grow((void**)&L.sel_d, L.sel_d_bytes, sizeof(uint64_t) * (size_t)B * slice_slots(L.V, k)) ||
        !grow((void**)&L.sel_i, L.sel_i_bytes, sizeof(int32_t) * (size_t)B * slice_slots(L.V, k))) {
        err = "vocab lattice: device allocation failed";
        return SLX_EOOM;
    }
    return SLX_OK;
}

int query_topk(Lattice& L, int B, int k, int32_t* d_ids, uint64_t* d_dist, cudaStream_t st) {
    if (B <= 0 || k <= 0) return 0;
    const int keff = (int64_t)k > L.V ? (int)L.V : k;
    const int64_t total = (int64_t)B * L.d;
    int n = 0;
    if (total > 0) {
        k_vocab_quantize<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(L.hf, total, L.hq);
        n++;
    }
    if (keff > 0) {
        n += candidates(L, B, keff, d_dist != nullptr, st);
        cudaMemcpy2DAsync(d_ids, sizeof(int32_t) * k, L.cand, sizeof(int32_t) * keff, sizeof(int32_t) * keff, B,
                          cudaMemcpyDeviceToDevice, st);
        if (d_dist)
            cudaMemcpy2DAsync(d_dist, sizeof(uint64_t) * k, L.cdist, sizeof(uint64_t) * keff, sizeof(uint64_t) * keff, B,
                              cudaMemcpyDeviceToDevice, st);
    }
    if (k > keff) {  // past the vocabulary: id -1, distance UINT64_MAX
        cudaMemset2DAsync((uint8_t*)d_ids + sizeof(int32_t) * keff, sizeof(int32_t) * k, 0xFF,
                          sizeof(int32_t) * (k - keff), B, st);
        if (d_dist)
            cudaMemset2DAsync((uint8_t*)d_dist + sizeof(uint64_t) * keff, sizeof(uint64_t) * k, 0xFF,
                              sizeof(uint64_t) * (k - keff), B, st);
    }
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
    if (keff > 0) n += candidates(L, B, keff, false, st);
    const size_t smem = sizeof(float) * (size_t)L.d;
    slx::ensure_smem((const void*)k_vocab_score, smem);
    k_vocab_score<<<(unsigned)B, ST, smem, st>>>(L.table, L.d, L.hf, L.cand, keff, eos, d_next);
    return n + 1;
}

}  // namespace vocab
}  // namespace slx
