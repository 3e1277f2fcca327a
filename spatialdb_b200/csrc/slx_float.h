// slx_float.h -- TransformerEmbeddingSource, the fp32 twin of the encoder (k_float.cu).
#pragma once
#include <cstddef>
#include <cstdint>
#include <vector>

#include <cuda_runtime.h>

namespace slx {
namespace fenc {

struct Layer {
    const float *qkv = nullptr, *o = nullptr, *up = nullptr, *gate = nullptr, *down = nullptr;  // [out][in]
    const float *anw = nullptr, *anb = nullptr, *lnw = nullptr, *lnb = nullptr;
};

struct Model {
    int d = 0, heads = 0, ff = 0, unk = 0;
    const float* tok = nullptr;  // [tok_rows][d]
    int64_t tok_rows = 0;
    const float *tt = nullptr, *enw = nullptr, *enb = nullptr;
    const float *cos = nullptr, *sin = nullptr;  // [512][hd / 2] RopeCache
    std::vector<Layer> layers;
};

struct Workspace {
    float *x = nullptr, *qkv = nullptr, *att = nullptr, *h = nullptr, *up = nullptr, *gate = nullptr, *sc = nullptr;
    size_t cx = 0, cqkv = 0, catt = 0, ch = 0, cup = 0, cgate = 0, csc = 0;
    void release();
};

// L2-normalised mean-pooled embeddings d_out[B][d] of B sequences of T ids. Returns the kernels
// launched, or -1 when the workspace could not be allocated.
int forward(const Model& m, const int32_t* d_ids, int B, int T, float* d_out, Workspace& ws, cudaStream_t st,
            int64_t* launches);

}  // namespace fenc
}  // namespace slx
