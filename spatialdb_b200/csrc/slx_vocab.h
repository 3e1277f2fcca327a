// slx_vocab.h -- the VocabLattice lm-head of the causal LM (k_vocab.cu).
#pragma once
#include <cstdint>
#include <string>

#include <cuda_runtime.h>

#include "slx_kernels.h"

namespace slx {
namespace vocab {

constexpr int KMAX = 8192;  // largest k one query block selects and sorts

struct Lattice {
    int64_t V = 0;               // rows: min(vocab, token-table rows)
    int d = 0;
    uint16_t* table = nullptr;   // [V][d] Half bits of the token rows (TokenEmbeddingsFloat is their float)
    uint64_t* en = nullptr;      // [V] sum of the quantized row's squares mod 2^64
    // per-query scratch, grown to the largest batch seen
    int64_t* hq = nullptr;       // [B][d] hidden states quantized with VocabLattice's options
    float* hf = nullptr;         // [B][d] hidden states as float
    uint64_t* hn = nullptr;      // [B] sum of hq^2 mod 2^64
    uint64_t* dist = nullptr;    // [B][V]
    int32_t* cand = nullptr;     // [B][k] nearest rows, ascending (distance, row)
    uint64_t* cdist = nullptr;   // [B][k] their distances
    uint64_t* sel_d = nullptr;   // [B][slices][k] per-slice candidates (distance)
    int32_t* sel_i = nullptr;    // [B][slices][k] per-slice candidates (row)
    size_t hq_bytes = 0, hf_bytes = 0, hn_bytes = 0, dist_bytes = 0, cand_bytes = 0, cdist_bytes = 0;
    size_t sel_d_bytes = 0, sel_i_bytes = 0;
};

// Builds the lattice's table from the causal model's token tensor (once per model).
int build(const WDesc& tok, int64_t vocab, int d, Lattice& L, cudaStream_t st, std::string& err);
void release(Lattice& L);

// Scratch for B queries of k candidates; the float hidden states then go to L.hf.
int reserve(Lattice& L, int B, int k, std::string& err);

// VocabLattice.QueryTopK for the B float hidden states in L.hf: d_ids[B][k] in ascending
// (distance, row) order, -1 past the vocabulary (k > V); d_dist (nullable) [B][k] their distances,
// UINT64_MAX past the vocabulary. Returns the kernels launched.
int query_topk(Lattice& L, int B, int k, int32_t* d_ids, uint64_t* d_dist, cudaStream_t st);

// PredictNextToken with the lattice for B last hidden states (Q30 int64 [B][d]) -> d_next[B].
// k <= 0 gives eos (an empty candidate list). Returns the kernels launched.
int next_tokens(Lattice& L, const int64_t* d_last, int B, int scale_bits, int k, int eos, int32_t* d_next,
                cudaStream_t st);

}  // namespace vocab
}  // namespace slx
