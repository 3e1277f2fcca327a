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
    // the same weights split for the tensor-core projections (tc_prepare_weight), or null
    const float *qkv_t = nullptr, *o_t = nullptr, *up_t = nullptr, *gate_t = nullptr, *down_t = nullptr;
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
    float* planes = nullptr;  // the tensor-core projections' activation planes
    size_t cx = 0, cqkv = 0, catt = 0, ch = 0, cup = 0, cgate = 0, csc = 0, cplanes = 0;
    int* err = nullptr;  // device error word (bounded-wait timeouts), the context's
    void release();
};

// Tensor-core projections (k_fgemm_tc.cu): c[M][N] = a[M][K] . w[N][K]^T in fp32 from three tf32
// products of the operands split into high and low parts. tc_prepare_weight writes a weight's
// planes (tc_weight_bytes) once; tc_project splits the activations into act_planes
// (tc_act_bytes) and runs the GEMM. Both return false when nothing was queued.
size_t tc_weight_bytes(int N, int K);
bool tc_prepare_weight(const float* w, int N, int K, float* planes, cudaStream_t st);
size_t tc_act_bytes(int M, int K);
bool tc_project(const float* a, int M, int K, const float* w_planes, int N, float* c, float* act_planes, int* err,
                cudaStream_t st);

// L2-normalised mean-pooled embeddings d_out[B][d] of B sequences of T ids. Returns the kernels
// launched, or -1 when the workspace could not be allocated.
int forward(const Model& m, const int32_t* d_ids, int B, int T, float* d_out, Workspace& ws, cudaStream_t st,
            int64_t* launches);

}  // namespace fenc
}  // namespace slx
