// k_tree.cu -- EmbeddingLatticeBuilder (Lattice/EmbeddingLatticeBuilder.cs:11-127) on the device, and
// SparseLatticeSerializer (Lattice/SparseLatticeSerializer.cs:5-195) with Int32 payloads.
//
// The reference recurses: a span of more than LeafThreshold occupants is split at the median of its
// highest-variance dimension (variance sumSq * N - sum^2 over the span, among dimensions some
// occupant populates; median sorted[N / 2]; a two-pointer partition moves values below the median
// to the left), and becomes a leaf when no dimension is populated or a side would be empty. Here
// every span of one tree level is processed together:
//   k_stats (+ k_stats_reduce for spans longer than one work item): per dimension sum, Int128 sum of
//     squares and population over the span's rows, then the best dimension (equal variances: the
//     lowest dimension; the reference's choice follows ConcurrentDictionary enumeration order);
//   k_gather: the split dimension's value of every occupant;
//   k_sel_hist / k_sel_pick: an MSB-first radix select of the (N/2)-th smallest value per span;
//   k_part_*: the partition. The reference's loop swaps the i-th element >= median counted from the
//     left with the i-th element < median counted from the right, for as long as the first lies left
//     of the second; the pairs are exactly the elements >= median left of the boundary (the count of
//     values below the median) and those < median right of it, ranked from each end. A segmented
//     scan ranks them and each takes its partner's row, so leaves hold the reference's order.
// Work items are chunks of at most CH occupants of one span; the host keeps the node list and the
// next level's spans (one small read-back per level).
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "slx_status.h"
#include "slx_tree.h"

namespace slx {
namespace tree {
namespace {

using u128 = unsigned __int128;
using i128 = __int128;

constexpr int CH = 4096;  // occupants per work item
constexpr int BT = 256;   // threads per block
constexpr int DPT = 4;    // dimensions per thread per pass

struct LevelArgs {
    const int32_t* seg_start;
    const int32_t* seg_len;
    const int32_t* seg_nitems;
    const int32_t* item_seg;
    const int32_t* item_begin;
    const int32_t* item_len;
    const int32_t* item_pidx;  // partial slot of items of multi-item spans, -1 otherwise
    int32_t* best_dim;
    int32_t* pivot;
    int32_t* boundary;
    uint32_t* prefix;
    int32_t* krem;
    uint32_t* hist;      // [S][256]
    int32_t* item_cnt;
    int32_t* item_off;
    int64_t* psum;       // [P][dim]
    uint64_t* psq;       // [P][dim][2]
    uint8_t* ppop;       // [P][dim]
};

struct Best {
    u128 var;
    int dim;
};
__device__ __forceinline__ bool better(u128 v, int d, const Best& b) {
    return b.dim < 0 || v > b.var || (v == b.var && d < b.dim);
}

// Block-wide best (variance, dimension) of the threads' candidates; valid in thread 0.
__device__ Best block_best(Best mine, u128* s_var, int* s_dim) {
    s_var[threadIdx.x] = mine.var;
    s_dim[threadIdx.x] = mine.dim;
    __syncthreads();
    Best b{0, -1};
    if (threadIdx.x == 0)
        for (int t = 0; t < BT; t++)
            if (s_dim[t] >= 0 && better(s_var[t], s_dim[t], b)) b = Best{s_var[t], s_dim[t]};
    __syncthreads();
    return b;
}

__global__ void k_iota(int32_t* perm, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        perm[i] = (int32_t)i;
}

__global__ void __launch_bounds__(BT) k_stats(const int32_t* __restrict__ vals, int dim,
                                              const int32_t* __restrict__ perm, LevelArgs a) {
    __shared__ int32_t rows[CH];
    __shared__ u128 s_var[BT];
    __shared__ int s_dim[BT];
    const int item = blockIdx.x, tid = threadIdx.x;
    const int s = a.item_seg[item];
    const int64_t base = (int64_t)a.seg_start[s] + a.item_begin[item];
    const int len = a.item_len[item];
    const int64_t N = a.seg_len[s];
    const bool single = a.seg_nitems[s] == 1;
    const int pidx = a.item_pidx[item];
    for (int i = tid; i < len; i += BT) rows[i] = perm[base + i];
    __syncthreads();
    Best mine{0, -1};
    for (int d0 = 0; d0 < dim; d0 += BT * DPT) {
        int64_t sum[DPT];
        u128 sq[DPT];
        bool pop[DPT];
#pragma unroll
        for (int t = 0; t < DPT; t++) {
            sum[t] = 0;
            sq[t] = 0;
            pop[t] = false;
        }
        for (int i = 0; i < len; i++) {
            const int32_t* r = vals + (int64_t)rows[i] * dim;
#pragma unroll
            for (int t = 0; t < DPT; t++) {
                const int d = d0 + t * BT + tid;
                if (d < dim) {
                    const int64_t v = r[d];
                    sum[t] += v;
                    sq[t] += (u128)(uint64_t)(v * v);
                    pop[t] |= v != 0;
                }
            }
        }
#pragma unroll
        for (int t = 0; t < DPT; t++) {
            const int d = d0 + t * BT + tid;
            if (d >= dim) continue;
            if (single) {
                if (pop[t]) {
                    const u128 var = (u128)((i128)sq[t] * N - (i128)sum[t] * sum[t]);
                    if (better(var, d, mine)) mine = Best{var, d};
                }
            } else {
                const int64_t o = (int64_t)pidx * dim + d;
                a.psum[o] = sum[t];
                a.psq[2 * o] = (uint64_t)sq[t];
                a.psq[2 * o + 1] = (uint64_t)(sq[t] >> 64);
                a.ppop[o] = pop[t];
            }
        }
    }
    if (single) {
        const Best b = block_best(mine, s_var, s_dim);
        if (tid == 0) a.best_dim[s] = b.dim;
    }
}

// Spans of several work items: sum their partials. mseg lists those spans, item0 their first item.
__global__ void __launch_bounds__(BT) k_stats_reduce(int dim, const int32_t* __restrict__ mseg,
                                                     const int32_t* __restrict__ item0, LevelArgs a) {
    __shared__ u128 s_var[BT];
    __shared__ int s_dim[BT];
    const int s = mseg[blockIdx.x];
    const int it0 = item0[blockIdx.x], nit = a.seg_nitems[s];
    const int p0 = a.item_pidx[it0];
    const int64_t N = a.seg_len[s];
    Best mine{0, -1};
    for (int d = threadIdx.x; d < dim; d += BT) {
        int64_t sum = 0;
        u128 sq = 0;
        bool pop = false;
        for (int j = 0; j < nit; j++) {
            const int64_t o = (int64_t)(p0 + j) * dim + d;
            sum += a.psum[o];
            sq += ((u128)a.psq[2 * o + 1] << 64) | a.psq[2 * o];
            pop |= a.ppop[o] != 0;
        }
        if (pop) {
            const u128 var = (u128)((i128)sq * N - (i128)sum * sum);
            if (better(var, d, mine)) mine = Best{var, d};
        }
    }
    const Best b = block_best(mine, s_var, s_dim);
    if (threadIdx.x == 0) a.best_dim[s] = b.dim;
}

__global__ void k_gather(const int32_t* __restrict__ vals, int dim, const int32_t* __restrict__ perm,
                         int32_t* __restrict__ pv, LevelArgs a) {
    const int item = blockIdx.x;
    const int s = a.item_seg[item];
    const int bd = a.best_dim[s];
    if (bd < 0) return;
    const int64_t base = (int64_t)a.seg_start[s] + a.item_begin[item];
    const int len = a.item_len[item];
    for (int i = threadIdx.x; i < len; i += blockDim.x) pv[base + i] = vals[(int64_t)perm[base + i] * dim + bd];
}

__global__ void k_sel_init(int S, LevelArgs a) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= S) return;
    a.prefix[s] = 0;
    a.krem[s] = a.seg_len[s] / 2 + 1;  // 1-based rank of sorted[N / 2]
}

// Radix select, one byte per round (round 3 = most significant) of the order-preserving key v ^ 2^31.
__global__ void __launch_bounds__(BT) k_sel_hist(const int32_t* __restrict__ pv, int round, LevelArgs a) {
    __shared__ unsigned h[256];
    const int item = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
    const int s = a.item_seg[item];
    if (a.best_dim[s] < 0) return;
    for (int b = tid; b < 256; b += BT) h[b] = 0;
    __syncthreads();
    const int64_t base = (int64_t)a.seg_start[s] + a.item_begin[item];
    const int len = a.item_len[item];
    const uint32_t pre = a.prefix[s];
    const uint32_t mask = round == 3 ? 0u : 0xFFFFFFFFu << (8 * (round + 1));
    for (int i0 = 0; i0 < len; i0 += BT) {
        const int i = i0 + tid;
        unsigned bin = 256;
        if (i < len) {
            const uint32_t key = (uint32_t)pv[base + i] ^ 0x80000000u;
            if ((key & mask) == pre) bin = (key >> (8 * round)) & 255u;
        }
        const unsigned same = __match_any_sync(0xffffffffu, bin);
        if (bin < 256 && lane == __ffs(same) - 1) atomicAdd(&h[bin], (unsigned)__popc(same));
    }
    __syncthreads();
    for (int b = tid; b < 256; b += BT)
        if (h[b]) atomicAdd(&a.hist[(int64_t)s * 256 + b], h[b]);
}

__global__ void k_sel_pick(int S, int round, LevelArgs a) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= S || a.best_dim[s] < 0) return;
    uint32_t* h = a.hist + (int64_t)s * 256;
    const int k = a.krem[s];
    int below = 0, b = 0;
    for (; b < 255; b++) {
        if (below + (int)h[b] >= k) break;
        below += (int)h[b];
    }
    a.prefix[s] |= (uint32_t)b << (8 * round);
    a.krem[s] = k - below;
    for (int j = 0; j < 256; j++) h[j] = 0;
    if (round == 0) a.pivot[s] = (int32_t)(a.prefix[s] ^ 0x80000000u);
}

// Thread t of an item owns its occupants t*PER .. t*PER+PER-1, so counts and scans keep span order.
constexpr int PER = CH / BT;

__device__ int block_excl_scan(int v, int* total) {
    __shared__ int ws[BT / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) ws[warp] = x;
    __syncthreads();
    int before = 0, all = 0;
    for (int w = 0; w < BT / 32; w++) {
        before += w < warp ? ws[w] : 0;
        all += ws[w];
    }
    __syncthreads();
    *total = all;
    return before + x - v;
}

__global__ void __launch_bounds__(BT) k_part_count(const int32_t* __restrict__ pv, LevelArgs a) {
    const int item = blockIdx.x, tid = threadIdx.x;
    const int s = a.item_seg[item];
    if (a.best_dim[s] < 0) return;
    const int64_t base = (int64_t)a.seg_start[s] + a.item_begin[item];
    const int len = a.item_len[item];
    const int32_t p = a.pivot[s];
    int c = 0;
    for (int u = 0; u < PER; u++) {
        const int i = tid * PER + u;
        c += (i < len && pv[base + i] < p) ? 1 : 0;
    }
    int tot;
    block_excl_scan(c, &tot);
    if (tid == 0) a.item_cnt[item] = tot;
}

__global__ void k_part_offsets(int S, const int32_t* __restrict__ seg_item0, LevelArgs a) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= S || a.best_dim[s] < 0) return;
    int off = 0;
    const int i0 = seg_item0[s], ni = a.seg_nitems[s];
    for (int j = 0; j < ni; j++) {
        a.item_off[i0 + j] = off;
        off += a.item_cnt[i0 + j];
    }
    a.boundary[s] = off;
}

// F[pos] = values below the pivot before pos in the span; the misplaced elements record their
// span-local index under their rank: left ones (>= pivot, left of the boundary) counted from the
// left in lpos, right ones (< pivot, right of it) counted from the right in rpos.
__global__ void __launch_bounds__(BT) k_part_ranks(const int32_t* __restrict__ pv, int32_t* __restrict__ F,
                                                   int32_t* __restrict__ lpos, int32_t* __restrict__ rpos,
                                                   LevelArgs a) {
    const int item = blockIdx.x, tid = threadIdx.x;
    const int s = a.item_seg[item];
    if (a.best_dim[s] < 0) return;
    const int64_t start = a.seg_start[s];
    const int b0 = a.item_begin[item];
    const int64_t base = start + b0;
    const int len = a.item_len[item];
    const int32_t p = a.pivot[s];
    const int bnd = a.boundary[s];
    bool f[PER];
    int c = 0;
#pragma unroll
    for (int u = 0; u < PER; u++) {
        const int i = tid * PER + u;
        f[u] = i < len && pv[base + i] < p;
        c += f[u];
    }
    int tot;
    int run = a.item_off[item] + block_excl_scan(c, &tot);
#pragma unroll
    for (int u = 0; u < PER; u++) {
        const int li = tid * PER + u;
        if (li >= len) break;
        const int i = b0 + li;  // span-local index
        F[base + li] = run;
        if (i < bnd && !f[u]) lpos[start + (i - run)] = i;
        if (i >= bnd && f[u]) rpos[start + (bnd - run - 1)] = i;
        run += f[u];
    }
}

__global__ void k_part_swap(const int32_t* __restrict__ pv, const int32_t* __restrict__ F,
                            const int32_t* __restrict__ lpos, const int32_t* __restrict__ rpos,
                            const int32_t* __restrict__ perm, int32_t* __restrict__ tmp, LevelArgs a) {
    const int item = blockIdx.x;
    const int s = a.item_seg[item];
    if (a.best_dim[s] < 0) return;
    const int64_t start = a.seg_start[s];
    const int b0 = a.item_begin[item];
    const int len = a.item_len[item];
    const int32_t p = a.pivot[s];
    const int bnd = a.boundary[s];
    for (int li = threadIdx.x; li < len; li += blockDim.x) {
        const int64_t pos = start + b0 + li;
        const int i = b0 + li;
        const bool f = pv[pos] < p;
        const int r = F[pos];
        int from = i;
        if (i < bnd && !f) from = rpos[start + (i - r)];
        else if (i >= bnd && f) from = lpos[start + (bnd - r - 1)];
        tmp[pos] = perm[start + from];
    }
}

__global__ void k_copy_back(const int32_t* __restrict__ tmp, int32_t* __restrict__ perm, LevelArgs a) {
    const int item = blockIdx.x;
    const int s = a.item_seg[item];
    if (a.best_dim[s] < 0) return;
    const int64_t base = (int64_t)a.seg_start[s] + a.item_begin[item];
    const int len = a.item_len[item];
    for (int i = threadIdx.x; i < len; i += blockDim.x) perm[base + i] = tmp[base + i];
}

// ---- SLAT occupant records --------------------------------------------------------------------
// Record of the occupant at leaf-order position p: int32 TotalDimensions, int32 entry count,
// (uint16 dimension, int64 value) per nonzero component in ascending dimension, int32 payload.

__global__ void k_rec_sizes(const int32_t* __restrict__ vals, int dim, const int32_t* __restrict__ perm, int64_t p0,
                            int64_t p1, int64_t* __restrict__ size) {
    const int lane = threadIdx.x & 31;
    for (int64_t p = p0 + (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / 32; p < p1;
         p += (int64_t)gridDim.x * blockDim.x / 32) {
        const int32_t* r = vals + (int64_t)perm[p] * dim;
        int nnz = 0;
        for (int d0 = 0; d0 < dim; d0 += 32) {
            const int d = d0 + lane;
            nnz += __popc(__ballot_sync(0xffffffffu, d < dim && r[d] != 0));
        }
        if (lane == 0) size[p - p0] = 12 + 10 * (int64_t)nnz;
    }
}

__device__ __forceinline__ void put_bytes(uint8_t* dst, uint64_t v, int n) {
    for (int b = 0; b < n; b++) dst[b] = (uint8_t)(v >> (8 * b));
}

__global__ void k_rec_write(const int32_t* __restrict__ vals, int dim, const int32_t* __restrict__ perm,
                            const int32_t* __restrict__ payload, int64_t p0, int64_t p1, const int64_t* __restrict__ off,
                            uint8_t* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    for (int64_t p = p0 + (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / 32; p < p1;
         p += (int64_t)gridDim.x * blockDim.x / 32) {
        const int32_t row = perm[p];
        const int32_t* r = vals + (int64_t)row * dim;
        uint8_t* dst = out + off[p - p0];
        int e = 0;
        for (int d0 = 0; d0 < dim; d0 += 32) {
            const int d = d0 + lane;
            const int32_t v = d < dim ? r[d] : 0;
            const unsigned m = __ballot_sync(0xffffffffu, v != 0);
            if (v != 0) {
                uint8_t* q = dst + 8 + 10 * (int64_t)(e + __popc(m & ((1u << lane) - 1)));
                put_bytes(q, (uint64_t)d, 2);
                put_bytes(q + 2, (uint64_t)(int64_t)v, 8);
            }
            e += __popc(m);
        }
        if (lane == 0) {
            put_bytes(dst, (uint64_t)(uint32_t)dim, 4);
            put_bytes(dst + 4, (uint64_t)(uint32_t)e, 4);
            put_bytes(dst + 8 + 10 * (int64_t)e, (uint64_t)(uint32_t)payload[row], 4);
        }
    }
}

template <class T>
bool grow(T*& p, size_t& cap, size_t count) {
    if (count == 0) count = 1;
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

struct Scratch {
    int32_t *seg_start = nullptr, *seg_len = nullptr, *seg_nitems = nullptr, *seg_item0 = nullptr;
    int32_t *item_seg = nullptr, *item_begin = nullptr, *item_len = nullptr, *item_pidx = nullptr;
    int32_t *best_dim = nullptr, *pivot = nullptr, *boundary = nullptr, *krem = nullptr;
    uint32_t *prefix = nullptr, *hist = nullptr;
    int32_t *item_cnt = nullptr, *item_off = nullptr, *mseg = nullptr, *mitem0 = nullptr;
    int64_t* psum = nullptr;
    uint64_t* psq = nullptr;
    uint8_t* ppop = nullptr;
    int32_t *pv = nullptr, *F = nullptr, *lpos = nullptr, *rpos = nullptr, *tmp = nullptr;
    size_t c_seg = 0, c_seg2 = 0, c_seg3 = 0, c_seg4 = 0, c_item = 0, c_item2 = 0, c_item3 = 0, c_item4 = 0;
    size_t c_bd = 0, c_pv = 0, c_bn = 0, c_kr = 0, c_pre = 0, c_hist = 0, c_cnt = 0, c_off = 0, c_ms = 0, c_mi = 0;
    size_t c_psum = 0, c_psq = 0, c_ppop = 0, c_pvv = 0, c_F = 0, c_l = 0, c_r = 0, c_t = 0;
    ~Scratch() {
        for (void* p : {(void*)seg_start, (void*)seg_len, (void*)seg_nitems, (void*)seg_item0, (void*)item_seg,
                        (void*)item_begin, (void*)item_len, (void*)item_pidx, (void*)best_dim, (void*)pivot,
                        (void*)boundary, (void*)krem, (void*)prefix, (void*)hist, (void*)item_cnt, (void*)item_off,
                        (void*)mseg, (void*)mitem0, (void*)psum, (void*)psq, (void*)ppop, (void*)pv, (void*)F,
                        (void*)lpos, (void*)rpos, (void*)tmp})
            cudaFree(p);
    }
};

struct Span {
    int64_t start, len;
    int node;
};
}  // namespace

void Sink::write(const void* p, size_t n) {
    if (!ok || n == 0) return;
    if (f) {
        ok = fwrite(p, 1, n, f) == n;
    } else if (mem) {
        if (used + n > cap) {
            ok = false;
            return;
        }
        memcpy(mem + used, p, n);
    }
    used += n;
}

void release(Tree& t) {
    cudaFree(t.perm);
    t = Tree();
}

int build(const int32_t* d_vals, int64_t n, int dim, int leaf_threshold, Tree& t, cudaStream_t st, std::string& err,
          int64_t* launches) {
    release(t);
    if (n < 0 || n > INT32_MAX - 1 || dim < 1 || dim > 65536) {
        err = "lattice tree: bad shape";
        return SLX_EINVAL;
    }
    t.n = n;
    if (cudaMalloc(&t.perm, sizeof(int32_t) * (size_t)std::max<int64_t>(n, 1)) != cudaSuccess) {
        cudaGetLastError();
        t.perm = nullptr;
        err = "lattice tree: device allocation failed";
        return SLX_EOOM;
    }
    int64_t nl = 0;
    if (n > 0) {
        k_iota<<<(unsigned)std::min<int64_t>((n + 255) / 256, 148 * 16), 256, 0, st>>>(t.perm, n);
        nl++;
    }
    auto make_node = [&](const Node& nd) {
        t.nodes.push_back(nd);
        return (int)t.nodes.size() - 1;
    };
    auto leaf = [&](int64_t start, int64_t count) {
        Node nd;
        nd.kind = 0;
        nd.start = start;
        nd.count = count;
        return nd;
    };
    t.root = make_node(leaf(0, n));
    std::vector<Span> active;
    if (n > leaf_threshold) active.push_back(Span{0, n, t.root});
    Scratch sc;
    // Upper bounds of every level's scratch, allocated once: active spans are disjoint and hold more
    // than leaf_threshold occupants each; work items number at most n / CH plus one per span, and
    // the items of multi-item spans at most 2 n / CH.
    if (!active.empty()) {
        const size_t smax = (size_t)(n / (leaf_threshold + 1) + 1);
        const size_t imax = (size_t)(n / CH) + smax + 1, pmax = (size_t)(2 * n / CH) + 2;
        if (!grow(sc.seg_start, sc.c_seg, smax) || !grow(sc.seg_len, sc.c_seg2, smax) ||
            !grow(sc.seg_nitems, sc.c_seg3, smax) || !grow(sc.seg_item0, sc.c_seg4, smax) ||
            !grow(sc.item_seg, sc.c_item, imax) || !grow(sc.item_begin, sc.c_item2, imax) ||
            !grow(sc.item_len, sc.c_item3, imax) || !grow(sc.item_pidx, sc.c_item4, imax) ||
            !grow(sc.best_dim, sc.c_bd, smax) || !grow(sc.pivot, sc.c_pv, smax) || !grow(sc.boundary, sc.c_bn, smax) ||
            !grow(sc.krem, sc.c_kr, smax) || !grow(sc.prefix, sc.c_pre, smax) || !grow(sc.hist, sc.c_hist, smax * 256) ||
            !grow(sc.item_cnt, sc.c_cnt, imax) || !grow(sc.item_off, sc.c_off, imax) || !grow(sc.mseg, sc.c_ms, smax) ||
            !grow(sc.mitem0, sc.c_mi, smax) || !grow(sc.psum, sc.c_psum, pmax * dim) ||
            !grow(sc.psq, sc.c_psq, pmax * dim * 2) || !grow(sc.ppop, sc.c_ppop, pmax * dim) ||
            !grow(sc.pv, sc.c_pvv, (size_t)n) || !grow(sc.F, sc.c_F, (size_t)n) || !grow(sc.lpos, sc.c_l, (size_t)n) ||
            !grow(sc.rpos, sc.c_r, (size_t)n) || !grow(sc.tmp, sc.c_t, (size_t)n)) {
            err = "lattice tree: device allocation failed";
            return SLX_EOOM;
        }
    }
    std::vector<int32_t> h_ss, h_sl, h_sn, h_si, h_is, h_ib, h_il, h_ip, h_ms, h_mi, h_bd, h_pv, h_bn;
    while (!active.empty()) {
        const int S = (int)active.size();
        h_ss.assign(S, 0);
        h_sl.assign(S, 0);
        h_sn.assign(S, 0);
        h_si.assign(S, 0);
        h_is.clear();
        h_ib.clear();
        h_il.clear();
        h_ip.clear();
        h_ms.clear();
        h_mi.clear();
        int npart = 0;
        for (int s = 0; s < S; s++) {
            const int64_t len = active[s].len;
            const int nit = (int)((len + CH - 1) / CH);
            h_ss[s] = (int32_t)active[s].start;
            h_sl[s] = (int32_t)len;
            h_sn[s] = nit;
            h_si[s] = (int32_t)h_is.size();
            if (nit > 1) {
                h_ms.push_back(s);
                h_mi.push_back((int32_t)h_is.size());
            }
            for (int c = 0; c < nit; c++) {
                h_is.push_back(s);
                h_ib.push_back(c * CH);
                h_il.push_back((int32_t)std::min<int64_t>(CH, len - (int64_t)c * CH));
                h_ip.push_back(nit > 1 ? npart++ : -1);
            }
        }
        const int I = (int)h_is.size(), M = (int)h_ms.size();
        if (!grow(sc.seg_start, sc.c_seg, S) || !grow(sc.seg_len, sc.c_seg2, S) || !grow(sc.seg_nitems, sc.c_seg3, S) ||
            !grow(sc.seg_item0, sc.c_seg4, S) || !grow(sc.item_seg, sc.c_item, I) || !grow(sc.item_begin, sc.c_item2, I) ||
            !grow(sc.item_len, sc.c_item3, I) || !grow(sc.item_pidx, sc.c_item4, I) || !grow(sc.best_dim, sc.c_bd, S) ||
            !grow(sc.pivot, sc.c_pv, S) || !grow(sc.boundary, sc.c_bn, S) || !grow(sc.krem, sc.c_kr, S) ||
            !grow(sc.prefix, sc.c_pre, S) || !grow(sc.hist, sc.c_hist, (size_t)S * 256) ||
            !grow(sc.item_cnt, sc.c_cnt, I) || !grow(sc.item_off, sc.c_off, I) || !grow(sc.mseg, sc.c_ms, M) ||
            !grow(sc.mitem0, sc.c_mi, M) || !grow(sc.psum, sc.c_psum, (size_t)npart * dim) ||
            !grow(sc.psq, sc.c_psq, (size_t)npart * dim * 2) || !grow(sc.ppop, sc.c_ppop, (size_t)npart * dim) ||
            !grow(sc.pv, sc.c_pvv, (size_t)n) || !grow(sc.F, sc.c_F, (size_t)n) || !grow(sc.lpos, sc.c_l, (size_t)n) ||
            !grow(sc.rpos, sc.c_r, (size_t)n) || !grow(sc.tmp, sc.c_t, (size_t)n)) {
            err = "lattice tree: device allocation failed";
            return SLX_EOOM;
        }
        auto up = [&](int32_t* d, const std::vector<int32_t>& h) {
            if (!h.empty()) cudaMemcpyAsync(d, h.data(), h.size() * 4, cudaMemcpyHostToDevice, st);
        };
        up(sc.seg_start, h_ss);
        up(sc.seg_len, h_sl);
        up(sc.seg_nitems, h_sn);
        up(sc.seg_item0, h_si);
        up(sc.item_seg, h_is);
        up(sc.item_begin, h_ib);
        up(sc.item_len, h_il);
        up(sc.item_pidx, h_ip);
        up(sc.mseg, h_ms);
        up(sc.mitem0, h_mi);
        cudaMemsetAsync(sc.hist, 0, (size_t)S * 256 * 4, st);
        LevelArgs a{sc.seg_start, sc.seg_len, sc.seg_nitems, sc.item_seg, sc.item_begin, sc.item_len, sc.item_pidx,
                    sc.best_dim, sc.pivot, sc.boundary, sc.prefix, sc.krem, sc.hist, sc.item_cnt, sc.item_off,
                    sc.psum, sc.psq, sc.ppop};
        const unsigned sg = (unsigned)((S + 255) / 256);
        k_stats<<<(unsigned)I, BT, 0, st>>>(d_vals, dim, t.perm, a);
        if (M > 0) k_stats_reduce<<<(unsigned)M, BT, 0, st>>>(dim, sc.mseg, sc.mitem0, a);
        k_gather<<<(unsigned)I, BT, 0, st>>>(d_vals, dim, t.perm, sc.pv, a);
        k_sel_init<<<sg, 256, 0, st>>>(S, a);
        for (int round = 3; round >= 0; round--) {
            k_sel_hist<<<(unsigned)I, BT, 0, st>>>(sc.pv, round, a);
            k_sel_pick<<<sg, 256, 0, st>>>(S, round, a);
        }
        k_part_count<<<(unsigned)I, BT, 0, st>>>(sc.pv, a);
        k_part_offsets<<<sg, 256, 0, st>>>(S, sc.seg_item0, a);
        k_part_ranks<<<(unsigned)I, BT, 0, st>>>(sc.pv, sc.F, sc.lpos, sc.rpos, a);
        k_part_swap<<<(unsigned)I, BT, 0, st>>>(sc.pv, sc.F, sc.lpos, sc.rpos, t.perm, sc.tmp, a);
        k_copy_back<<<(unsigned)I, BT, 0, st>>>(sc.tmp, t.perm, a);
        nl += 16 + (M > 0 ? 1 : 0);
        h_bd.resize(S);
        h_pv.resize(S);
        h_bn.resize(S);
        cudaMemcpyAsync(h_bd.data(), sc.best_dim, (size_t)S * 4, cudaMemcpyDeviceToHost, st);
        cudaMemcpyAsync(h_pv.data(), sc.pivot, (size_t)S * 4, cudaMemcpyDeviceToHost, st);
        cudaMemcpyAsync(h_bn.data(), sc.boundary, (size_t)S * 4, cudaMemcpyDeviceToHost, st);
        const cudaError_t e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) {
            err = std::string("lattice tree: ") + cudaGetErrorString(e);
            return SLX_ECUDA;
        }
        std::vector<Span> next;
        for (int s = 0; s < S; s++) {
            const Span sp = active[s];
            const int64_t bnd = h_bn[s];
            if (h_bd[s] < 0 || bnd == 0 || bnd == sp.len) continue;  // stays the leaf it was created as
            Node br;
            br.kind = 1;
            br.mask = 3;
            br.dim = h_bd[s];
            br.val = h_pv[s];
            const int below = make_node(leaf(sp.start, bnd));
            const int above = make_node(leaf(sp.start + bnd, sp.len - bnd));
            br.below = below;
            br.above = above;
            t.nodes[sp.node] = br;
            if (bnd > leaf_threshold) next.push_back(Span{sp.start, bnd, below});
            if (sp.len - bnd > leaf_threshold) next.push_back(Span{sp.start + bnd, sp.len - bnd, above});
        }
        active.swap(next);
    }
    if (launches) *launches += nl;
    return SLX_OK;
}

std::vector<int> preorder(const Tree& t) {
    std::vector<int> order, stack;
    if (t.root >= 0) stack.push_back(t.root);
    while (!stack.empty()) {
        const int i = stack.back();
        stack.pop_back();
        order.push_back(i);
        const Node& nd = t.nodes[i];
        if (nd.kind == 1) {  // below is visited first
            if (nd.above >= 0) stack.push_back(nd.above);
            if (nd.below >= 0) stack.push_back(nd.below);
        }
    }
    return order;
}

Stats stats(const Tree& t) {
    Stats s;
    std::vector<std::pair<int, int64_t>> stack;
    if (t.root >= 0) stack.push_back({t.root, 0});
    while (!stack.empty()) {
        const auto [i, depth] = stack.back();
        stack.pop_back();
        const Node& nd = t.nodes[i];
        s.nodes++;
        s.max_depth = std::max(s.max_depth, depth);
        if (nd.kind == 0) {
            s.leaves++;
            s.occupants += nd.count;
        } else {
            s.branches++;
            if (nd.above >= 0) stack.push_back({nd.above, depth + 1});
            if (nd.below >= 0) stack.push_back({nd.below, depth + 1});
        }
    }
    return s;
}

int slat_size(const Tree& t, const int32_t* d_vals, int dim, int64_t* size, cudaStream_t st, std::string& err,
              int64_t* launches) {
    int64_t total = 6;
    for (const Node& nd : t.nodes) total += nd.kind == 1 ? 12 : 5;
    if (t.n > 0) {
        int64_t* d_size = nullptr;
        if (cudaMalloc(&d_size, sizeof(int64_t) * t.n) != cudaSuccess) {
            cudaGetLastError();
            err = "slat: device allocation failed";
            return SLX_EOOM;
        }
        k_rec_sizes<<<(unsigned)std::min<int64_t>((t.n + 7) / 8, 148 * 32), 256, 0, st>>>(d_vals, dim, t.perm, 0, t.n,
                                                                                          d_size);
        std::vector<int64_t> h((size_t)t.n);
        cudaMemcpyAsync(h.data(), d_size, sizeof(int64_t) * t.n, cudaMemcpyDeviceToHost, st);
        const cudaError_t e = cudaStreamSynchronize(st);
        cudaFree(d_size);
        if (e != cudaSuccess) {
            err = cudaGetErrorString(e);
            return SLX_ECUDA;
        }
        for (int64_t v : h) total += v;
        if (launches) *launches += 1;
    }
    *size = total;
    return SLX_OK;
}

int save(const Tree& t, const int32_t* d_vals, int dim, const int32_t* d_payload, Sink& out, cudaStream_t st,
         std::string& err, int64_t* launches, size_t batch_bytes) {
    const int64_t n = t.n;
    // record sizes of every leaf-order position
    std::vector<int64_t> size((size_t)n);
    int64_t* d_size = nullptr;
    uint8_t* d_buf = nullptr;
    int64_t* d_off = nullptr;
    auto fail = [&](int code, const char* msg) {
        cudaFree(d_size);
        cudaFree(d_buf);
        cudaFree(d_off);
        cudaGetLastError();
        err = msg;
        return code;
    };
    int64_t nl = 0;
    if (n > 0) {
        if (cudaMalloc(&d_size, sizeof(int64_t) * n) != cudaSuccess) return fail(SLX_EOOM, "slat: device allocation failed");
        k_rec_sizes<<<(unsigned)std::min<int64_t>((n + 7) / 8, 148 * 32), 256, 0, st>>>(d_vals, dim, t.perm, 0, n, d_size);
        nl++;
        cudaMemcpyAsync(size.data(), d_size, sizeof(int64_t) * n, cudaMemcpyDeviceToHost, st);
        if (cudaStreamSynchronize(st) != cudaSuccess) return fail(SLX_ECUDA, "slat: record sizes failed");
    }
    // batches of consecutive positions, each at most batch_bytes of records (at least one record)
    std::vector<int64_t> bstart{0};
    {
        int64_t acc = 0;
        for (int64_t p = 0; p < n; p++) {
            if (acc > 0 && acc + size[p] > (int64_t)batch_bytes) {
                bstart.push_back(p);
                acc = 0;
            }
            acc += size[p];
        }
        bstart.push_back(n);
    }
    int64_t max_batch = 0, max_count = 0;
    for (size_t b = 0; b + 1 < bstart.size(); b++) {
        int64_t bytes = 0;
        for (int64_t p = bstart[b]; p < bstart[b + 1]; p++) bytes += size[p];
        max_batch = std::max(max_batch, bytes);
        max_count = std::max(max_count, bstart[b + 1] - bstart[b]);
    }
    uint8_t* host = nullptr;  // pinned staging of one batch of records
    std::vector<int64_t> off;
    if (n > 0) {
        if (cudaMalloc(&d_buf, (size_t)std::max<int64_t>(max_batch, 1)) != cudaSuccess ||
            cudaMalloc(&d_off, sizeof(int64_t) * (size_t)std::max<int64_t>(max_count, 1)) != cudaSuccess ||
            cudaMallocHost(&host, (size_t)std::max<int64_t>(max_batch, 1)) != cudaSuccess) {
            cudaFreeHost(host);
            return fail(SLX_EOOM, "slat: allocation failed");
        }
        off.resize((size_t)max_count);
    }
    size_t cur = 0;          // batch index loaded in `host`
    bool loaded = false;
    int64_t bp0 = 0, bp1 = 0;
    auto load_batch = [&](size_t b) -> int {
        bp0 = bstart[b];
        bp1 = bstart[b + 1];
        int64_t acc = 0;
        for (int64_t p = bp0; p < bp1; p++) {
            off[p - bp0] = acc;
            acc += size[p];
        }
        cudaMemcpyAsync(d_off, off.data(), sizeof(int64_t) * (bp1 - bp0), cudaMemcpyHostToDevice, st);
        k_rec_write<<<(unsigned)std::min<int64_t>((bp1 - bp0 + 7) / 8, 148 * 32), 256, 0, st>>>(
            d_vals, dim, t.perm, d_payload, bp0, bp1, d_off, d_buf);
        nl++;
        cudaMemcpyAsync(host, d_buf, (size_t)acc, cudaMemcpyDeviceToHost, st);
        if (cudaStreamSynchronize(st) != cudaSuccess) return SLX_ECUDA;
        cur = b;
        loaded = true;
        return SLX_OK;
    };
    const uint32_t magic = 0x544C4153u;
    const uint16_t version = 1;
    out.write(&magic, 4);
    out.write(&version, 2);
    for (int i : preorder(t)) {
        const Node& nd = t.nodes[i];
        if (nd.kind == 1) {
            uint8_t h[12];
            h[0] = 1;
            const uint16_t d = (uint16_t)nd.dim;
            memcpy(h + 1, &d, 2);
            memcpy(h + 3, &nd.val, 8);
            h[11] = (uint8_t)nd.mask;
            out.write(h, 12);
            continue;
        }
        uint8_t h[5];
        h[0] = 0;
        const int32_t c = (int32_t)nd.count;
        memcpy(h + 1, &c, 4);
        out.write(h, 5);
        int64_t p = nd.start;
        const int64_t end = nd.start + nd.count;
        while (p < end) {
            if (!loaded || p >= bp1) {
                size_t b = loaded ? cur + 1 : 0;
                while (bstart[b + 1] <= p) b++;
                if (load_batch(b)) {
                    cudaFreeHost(host);
                    return fail(SLX_ECUDA, "slat: record kernel failed");
                }
            }
            const int64_t q = std::min(end, bp1);
            const int64_t from = off[p - bp0];
            const int64_t to = q < bp1 ? off[q - bp0] : off[bp1 - 1 - bp0] + size[bp1 - 1];
            out.write(host + from, (size_t)(to - from));
            p = q;
        }
    }
    cudaFree(d_size);
    cudaFree(d_buf);
    cudaFree(d_off);
    cudaFreeHost(host);
    if (launches) *launches += nl;
    if (!out.ok) {
        err = "slat: write failed";
        return SLX_EINVAL;
    }
    return SLX_OK;
}

namespace {
struct Reader {
    const uint8_t* p;
    int64_t n, pos = 0;
    int status = SLX_OK;
    std::string msg;
    template <class T> bool get(T& v) {
        if (status) return false;
        if (pos + (int64_t)sizeof(T) > n) {
            status = SLX_EEOF;
            msg = "Unable to read beyond the end of the stream.";
            return false;
        }
        memcpy(&v, p + pos, sizeof(T));
        pos += sizeof(T);
        return true;
    }
    bool fail(int code, std::string m) {
        status = code;
        msg = std::move(m);
        return false;
    }
};

int read_node(Reader& r, Loaded& out, int depth) {
    if (depth > 100000) {
        r.fail(SLX_EFORMAT, "SLAT tree deeper than 100000 levels");
        return -1;
    }
    uint8_t tag;
    if (!r.get(tag)) return -1;
    if (tag == 0) {
        int32_t count;
        if (!r.get(count)) return -1;
        if (count < 0) {
            r.fail(SLX_EFORMAT, "negative leaf occupant count");
            return -1;
        }
        Node nd;
        nd.kind = 0;
        nd.start = (int64_t)out.payload.size();
        nd.count = count;
        for (int32_t i = 0; i < count; i++) {
            int32_t total, entries;
            if (!r.get(total) || !r.get(entries)) return -1;
            if (total <= 0) {
                r.fail(SLX_EINVAL, "Specified argument was out of the range of valid values. (Parameter 'totalDimensions')");
                return -1;
            }
            if (entries < 0) {
                r.fail(SLX_EFORMAT, "negative entry count");
                return -1;
            }
            if (out.dim == 0) {
                if (total > 16384) {
                    r.fail(SLX_EUNSUPPORTED, "SLAT occupants wider than 16384 dimensions");
                    return -1;
                }
                out.dim = total;
            }
            if (total != out.dim) {
                r.fail(SLX_EUNSUPPORTED, "SLAT occupants of different TotalDimensions");
                return -1;
            }
            const size_t row = out.payload.size();
            out.rows.resize((row + 1) * (size_t)total, 0);
            int prev = -1;
            for (int32_t e = 0; e < entries; e++) {
                uint16_t d;
                int64_t v;
                if (!r.get(d) || !r.get(v)) return -1;
                if ((int)d >= total) {
                    r.fail(SLX_EINVAL, "Entry dimension exceeds total dimensions.");
                    return -1;
                }
                if (v == 0) {
                    r.fail(SLX_EINVAL, "Sparse entry has value zero; zero entries must be omitted.");
                    return -1;
                }
                if ((int)d <= prev) {
                    r.fail(SLX_EINVAL, "Entries must be sorted ascending by dimension with no duplicates.");
                    return -1;
                }
                if (v < INT32_MIN || v > INT32_MAX) {
                    r.fail(SLX_ERANGE, "a SLAT component does not fit 32 bits");
                    return -1;
                }
                prev = d;
                out.rows[row * total + d] = (int32_t)v;
            }
            int32_t pay;
            if (!r.get(pay)) return -1;
            out.payload.push_back(pay);
        }
        out.nodes.push_back(nd);
        return (int)out.nodes.size() - 1;
    }
    if (tag == 1) {
        uint16_t d;
        int64_t v;
        uint8_t mask;
        if (!r.get(d) || !r.get(v) || !r.get(mask)) return -1;
        Node br;
        br.kind = 1;
        br.dim = d;
        br.val = v;
        br.mask = mask & 3;
        out.nodes.push_back(br);
        const int id = (int)out.nodes.size() - 1;
        int below = -1, above = -1;
        if (mask & 1) {
            below = read_node(r, out, depth + 1);
            if (below < 0) return -1;
        }
        if (mask & 2) {
            above = read_node(r, out, depth + 1);
            if (above < 0) return -1;
        }
        out.nodes[id].below = below;
        out.nodes[id].above = above;
        return id;
    }
    char m[64];
    snprintf(m, sizeof m, "Unknown node tag byte %u.", (unsigned)tag);
    r.fail(SLX_EFORMAT, m);
    return -1;
}
}  // namespace

int parse(const uint8_t* bytes, int64_t size, Loaded& out, std::string& err) {
    out = Loaded();
    Reader r{bytes, size};
    uint32_t magic;
    uint16_t version;
    if (!r.get(magic)) {
        err = r.msg;
        return r.status;
    }
    if (magic != 0x544C4153u) {
        char m[96];
        snprintf(m, sizeof m, "Invalid magic bytes: 0x%08X, expected 0x544C4153.", magic);
        err = m;
        return SLX_EFORMAT;
    }
    if (!r.get(version)) {
        err = r.msg;
        return r.status;
    }
    if (version != 1) {
        char m[96];
        snprintf(m, sizeof m, "Unsupported serialization version %u. Expected 1.", (unsigned)version);
        err = m;
        return SLX_EFORMAT;
    }
    out.root = read_node(r, out, 0);
    if (out.root < 0) {
        err = r.msg;
        return r.status ? r.status : SLX_EFORMAT;
    }
    if (out.payload.size() > (size_t)INT32_MAX - 256) {
        err = "SLAT file holds too many occupants";
        return SLX_EUNSUPPORTED;
    }
    return SLX_OK;
}

}  // namespace tree
}  // namespace slx
