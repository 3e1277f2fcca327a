// slx_search.h -- exact lattice k-NN search on the device (k_search.cu).
//
// SparseLattice's embed+search path quantizes float embeddings with EmbeddingAdapter.Quantize
// (Math/EmbeddingAdapter.cs:15-41; VocabLattice's options: ZeroThreshold 0.001, GlobalScale 1e9,
// no sparsity budget, Lattice/VocabLattice.cs:22-27) and returns the k nearest occupants by
// SparseVector.DistanceSquaredL2Fast (Math/SparseVector.cs:138-169) through EmbeddingLattice.
// QueryKNearestL2 (Lattice/EmbeddingLattice.cs:70-77). Here the database is a dense device array and
// every query is answered exactly: a tensor-core pass over the high parts of the components
// bounds every distance, and the few candidates it cannot rule out are re-scored exactly.
#pragma once
#include <cstdint>
#include <string>

#include <cuda_runtime.h>

namespace slx {
namespace search {

constexpr int T = 24;       // candidates kept per (query, slot)
constexpr int KMAX = 16;    // largest k: the bound needs candidates beyond the k-th
constexpr int MAX_DIM = 16384;

// Per-side statistics the bound needs, written by the quantize / split kernels.
struct SideStats {
    unsigned long long max_abs;    // max |component|
    unsigned long long max_norm2;  // max sum v^2 over rows (saturated at 2^63)
    unsigned long long max_h2;     // max sum v_h^2 over rows (v = v_h * 2^shift + v_l)
    unsigned long long max_l2;     // max sum v_l^2 over rows
    int range_bad;                 // a quantized component does not fit int32
    int pad[3];
};

struct Lattice {
    int device = 0;
    int64_t n = 0, npad = 0, id_base = 0;
    int dim = 0, dpad = 0;
    int32_t* vals = nullptr;     // [n][dim] quantized components
    int32_t* payload = nullptr;  // [n] ids of a lattice loaded from SLAT (query ids are payload[row])
    int8_t* planes = nullptr;    // [2][npad][dpad] balanced base-256 digits of the high parts
    uint64_t* norm2 = nullptr;   // [n] sum of squares
    SideStats* stats = nullptr;  // device
    alignas(64) unsigned char tmap[128];
    // query scratch, grown to the largest batch seen
    void* qws = nullptr;
    size_t qws_bytes = 0;
    void* xws = nullptr;  // exact re-scan scratch
    size_t xws_bytes = 0;
    int* counters = nullptr;  // [0] fallback count, [1] query range flag
};

// Builds the lattice from n float rows of dim components on the device. Returns 0 or an slx status.
int build(const float* d_vectors, int64_t n, int dim, float zero_threshold, int64_t global_scale, int64_t id_base,
          Lattice& L, cudaStream_t st, std::string& err);
// The same from rows already quantized to int32 (device [n][dim], copied).
int build_quantized(const int32_t* d_rows, int64_t n, int dim, int64_t id_base, Lattice& L, cudaStream_t st,
                    std::string& err);
void release(Lattice& L);

// k nearest rows for nq float queries: ids [nq][k] (id_base + row; -1 past the database) and
// distances [nq][k] (UINT64_MAX past the database), ascending (distance, id). exact_only skips the
// tensor-core bound and scans every row exactly. Synchronizes the stream once (fallback count).
int query(Lattice& L, const float* d_queries, int nq, int k, float zero_threshold, int64_t global_scale,
          bool exact_only, int64_t* d_ids, uint64_t* d_dist, int* n_fallback, cudaStream_t st, std::string& err,
          int64_t* launches);

// Merges `parts` ascending top-k lists per query ([parts][nq][k] each) into one ([nq][k]).
void merge_parts(const int64_t* ids, const uint64_t* dist, int parts, int nq, int k, int64_t* out_ids,
                 uint64_t* out_dist, cudaStream_t st);

}  // namespace search
}  // namespace slx
