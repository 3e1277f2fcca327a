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
    alignas(64) unsigned char tmap_w[128];  // CUtensorMap of the weight digit planes
    int8_t* row_shift = nullptr;              // device [N]: trailing zeros factored out of each row
};

// Bounded-wait settings of the tensor-core projection GEMM, per context.
struct WaitOptions {
    long long limit_cycles = 0;  // SM clock cycles before an mbarrier wait gives up (0: about two seconds)
    int stall_mma = 0;           // test hook: the MMA warp issues nothing, so the other warps' waits run out
};

// Per-model scratch shared by the projections.
struct GemmWorkspace {
    void* p = nullptr;
    size_t bytes = 0;
    int* err = nullptr;  // device error word (bounded-wait timeouts)
    unsigned tag = 0;    // last GEMV call's tag (the GEMV's overflow word is compared with it)
    const WaitOptions* wait = nullptr;  // the owning context's settings (nullptr: defaults)
    uint64_t gen = 0;    // bumped whenever p is reallocated (a captured CUDA graph holds p)
};

// Tensor-core kernel launchers (k_gemm_tc.cu).
namespace tc {
constexpr int BM = 128, BN = 64, BK = 128, LA = 5;  // padding of the digit planes (rows, weight rows, K bytes)
constexpr int GM = 32, GN = 128, GK = 128;        // projection tile: activation rows, weight rows, K bytes a stage
// Encodes a TMA map over int8 digit planes [batch][planes][rows][kpad] with a
// (box_k B, box_rows, planes, 1) box, 128-byte swizzle for box_k 128, 64-byte for box_k 64.
bool encode_planes(void* map128, void* base, int64_t kpad, int64_t rows, int planes, int box_rows, int64_t batch = 1,
                   int box_k = 128);
// Encodes a TMA map over `rows` rows of row_u16 16-bit elements (no swizzle), box (box_x, box_rows).
bool encode_rows_u16(void* map128, const void* base, int64_t row_u16, int64_t rows, int box_x, int box_rows);
// Per-row common trailing zeros of the Q30 composites -> tz[N].
void weight_tz(const WDesc& w, int8_t* tz, cudaStream_t st);
// Digits of the widest composite (after the optional per-row shift tz).
int weight_digits(const WDesc& w, cudaStream_t st, std::string& err, const int8_t* tz = nullptr);
void split_w(const WDesc& w, int lw, int64_t npad, int64_t kpad, int8_t* planes, cudaStream_t st,
             const int8_t* tz = nullptr);
void split_a(const int64_t* a, int64_t lda, int M, int K, int64_t mpad, int64_t kpad, int8_t* planes, int* overflow,
             cudaStream_t st);
// With a and w, a set *skip makes the kernel compute the exact product of a (int64 rows, lda) and
// w's composites on its CUDA cores instead (no separate fallback launch); without them it does nothing.
void launch(const void* tmap_a, const void* tmap_w, int lw, int M, int N, int K, int64_t mpad, int64_t npad, int64_t kpad,
            int shift, int64_t* c, int64_t ldc, const int64_t* r, int64_t ldr, const int* skip, int* err, cudaStream_t st,
            const int8_t* row_shift = nullptr, const WaitOptions* wait = nullptr, const int64_t* a = nullptr,
            int64_t lda = 0, const WDesc* w = nullptr);
// Per-head digit planes of rows at x + (b*T+t)*ld + h*hd -> [(b*nh+h)][LA][tpad][kpad].
// ApplyRoPE in place on the same head rows (cos / sin tables [T][hd/2], Q30), fused with their split;
// one launch for q (nh heads, tq padded rows) and k (nkv heads, tk padded rows).
void rope_split_heads(int64_t* q, int64_t ldq, int nh, int64_t tq, int8_t* qplanes, int64_t* k, int64_t ldk, int nkv,
                      int64_t tk, int8_t* kplanes, int B, int T, int hd, int64_t kpad, const int64_t* cs,
                      const int64_t* sn, int* overflow, cudaStream_t st, bool write_back = true);
void split_heads(const int64_t* x, int64_t ld, int B, int T, int nh, int hd, int64_t tpad, int64_t kpad, int8_t* planes,
                 int* overflow, cudaStream_t st);
}  // namespace tc

bool tc_enabled();
int gemm_prepare(const WDesc& w, GemmPlan& plan, cudaStream_t st, std::string& err);
int gemm_run(const int64_t* a, int64_t lda, int M, const WDesc& w, const GemmPlan& plan, int64_t* c, int64_t ldc,
              int shift, const int64_t* r, int64_t ldr, GemmWorkspace& ws, cudaStream_t st);
void gemm_workspace_free(GemmWorkspace& ws);
// gemm_run with the activations' digit planes already written by their producer: planes
// [5][round_up(M, 128)][plan.k_pad] int8 and its overflow word *flag (nonzero: the exact kernel
// computes the call). false (nothing queued) when the weight does not take the tensor-core path.
bool gemm_run_planes(const int8_t* planes, const int* flag, const int64_t* a, int64_t lda, int M, const WDesc& w,
                     const GemmPlan& plan, int64_t* c, int64_t ldc, int shift, const int64_t* r, int64_t ldr,
                     GemmWorkspace& ws, cudaStream_t st);
// Several projections of the same activations (Q/K/V, gate/up): c_i = (a . w_i^T) >> shift. The
// activation digits are formed once for all of them when every weight takes the tensor-core path
// with the same K padding; otherwise each runs as gemm_run. Returns the kernels queued.
int gemm_run_multi(const int64_t* a, int64_t lda, int M, int n, const WDesc* const* w, const GemmPlan* const* plan,
                   int64_t* const* c, const int64_t* ldc, int shift, GemmWorkspace& ws, cudaStream_t st);

// Decode-shaped exact GEMV (M <= 8) straight from packed Q4_0 / Q8_0 blocks with the long
// composite, digit products on the tensor cores (k_gemv_tc.cu).
bool gemv_supported(const WDesc& w, int M);
size_t gemv_workspace(int M, int N, int K);
// Grows ws for an M x N x K GEMV (zeroing it when it allocates); false when out of memory.
bool gemv_reserve(GemmWorkspace& ws, int M, int N, int K, cudaStream_t st);
// Single-row GEMV (k_gemv1.cu): one launch of persistent CTAs streaming the packed Q4_0 / Q8_0 rows
// by bulk copies, activation digits formed in-kernel. false (nothing queued) when the shape is not
// covered (K / 32 a multiple of 8 and at most 256, composite scale 2^24 .. 2^39, 16-byte aligned).
bool gemv1(const WDesc& w, const int64_t* a, int64_t* c, int shift, int* err, cudaStream_t st);
// One launch; bounded-wait timeouts set KERR_TIMEOUT in *ws.err when it is set.
int gemv_exact(const int64_t* a, int64_t lda, int M, const WDesc& w, int64_t* c, int64_t ldc, int shift,
               GemmWorkspace& ws, cudaStream_t st);

}  // namespace slx
