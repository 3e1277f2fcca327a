// slx_gemm.h -- projection GEMM dispatch: tensor-core limb GEMM when the operands' ranges allow it,
// exact CUDA-core GEMM otherwise. Both produce IntegerMatMul.MatMul's result bit for bit.
#pragma once
#include <cstdint>
#include <string>

#include <cuda_runtime.h>

#include "slx_kernels.h"

namespace slx {

// Load-time preparation of one weight for the tensor-core path.
struct GemmPlan {
    int use_tc = 0;          // tensor-core path available for this weight
    int wlimbs = 0;          // int8 limbs of the Q30 composite weight
    uint8_t* limbs = nullptr;  // device: limb planes [wlimbs][N_pad][K_pad]
    size_t limb_bytes = 0;
    int64_t n_pad = 0, k_pad = 0;
};

// Per-model scratch shared by the projections.
struct GemmWorkspace {
    void* p = nullptr;
    size_t bytes = 0;
};

int gemm_prepare(const WDesc& w, GemmPlan& plan, cudaStream_t st, std::string& err);
int gemm_run(const int64_t* a, int64_t lda, int M, const WDesc& w, const GemmPlan& plan, int64_t* c, int64_t ldc,
              int shift, const int64_t* r, int64_t ldr, GemmWorkspace& ws, cudaStream_t st);
void gemm_workspace_free(GemmWorkspace& ws);

}  // namespace slx
