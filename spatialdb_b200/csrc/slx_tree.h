// slx_tree.h -- the KD-tree lattice (EmbeddingLatticeBuilder) and its SLAT serialization (k_tree.cu).
#pragma once
#include <cstdint>
#include <string>
#include <vector>

#include <cuda_runtime.h>

namespace slx {
namespace tree {

// One node of the tree. Branch children are node indices (-1 when absent, which only a loaded
// SLAT file can produce); a leaf holds occupants perm[start .. start+count).
struct Node {
    int kind = 0;  // 0 leaf, 1 branch
    int mask = 0;  // branch: 1 below present, 2 above present
    int dim = 0;
    int64_t val = 0;
    int below = -1, above = -1;
    int64_t start = 0, count = 0;
};

struct Tree {
    std::vector<Node> nodes;
    int root = -1;
    int32_t* perm = nullptr;  // device [n]: row index of each leaf-order position
    int64_t n = 0;
};

struct Stats {
    int64_t nodes = 0, branches = 0, leaves = 0, occupants = 0, max_depth = 0;
};

// EmbeddingLatticeBuilder.Build over the n dense int32 rows d_vals[n][dim] (row i is occupant i).
int build(const int32_t* d_vals, int64_t n, int dim, int leaf_threshold, Tree& t, cudaStream_t st, std::string& err,
          int64_t* launches);
void release(Tree& t);
Stats stats(const Tree& t);
// Nodes in pre-order (the serializer's order).
std::vector<int> preorder(const Tree& t);

// Byte sink for the SLAT writer: a file or a caller buffer of `cap` bytes.
struct Sink {
    FILE* f = nullptr;
    uint8_t* mem = nullptr;
    size_t cap = 0, used = 0;
    bool ok = true;
    void write(const void* p, size_t n);
};

// Size in bytes of the tree's SLAT serialization (record sizes counted on the device).
int slat_size(const Tree& t, const int32_t* d_vals, int dim, int64_t* size, cudaStream_t st, std::string& err,
              int64_t* launches);

// SparseLatticeSerializer.Save with Int32 payloads: occupant records are produced on the device
// (rows d_vals in leaf order, nonzero components ascending, payload[row]) in batches of at most
// batch_bytes and stitched between the node headers on the host.
int save(const Tree& t, const int32_t* d_vals, int dim, const int32_t* d_payload, Sink& out, cudaStream_t st,
         std::string& err, int64_t* launches, size_t batch_bytes = (size_t)64 << 20);

// SparseLatticeSerializer.Load with Int32 payloads into dense rows (file order), payloads and the
// tree (perm = identity, set by the caller). Returns an slx status; rows must share one width and
// their values must fit int32 (SLX_ERANGE otherwise).
struct Loaded {
    std::vector<Node> nodes;
    int root = -1;
    std::vector<int32_t> rows;     // [n][dim]
    std::vector<int32_t> payload;  // [n]
    int dim = 0;
};
int parse(const uint8_t* bytes, int64_t size, Loaded& out, std::string& err);

}  // namespace tree
}  // namespace slx
