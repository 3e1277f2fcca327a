// gemm_dispatch.cu -- chooses the kernel for each projection (see slx_gemm.h).
//
// Tensor-core path (k_gemm_tc.cu) when the weight's Q30 composites fit 4 balanced int8 digits and
// K < 32768; per call the activations are split into 5 digit planes, and if any activation needs
// more digits the exact CUDA-core kernel (launched right behind, gated on the same device flag)
// computes the result instead. Either way the output equals IntegerMatMul.MatMul bit for bit.
#include <cstdlib>

#include "slx_gemm.h"
#include "slx_status.h"

namespace slx {

namespace {
int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }
}  // namespace

bool tc_enabled() {
    static int on = -1;
    if (on < 0) {
        const char* e = getenv("SLX_DISABLE_TC");
        on = (e && e[0] == '1') ? 0 : 1;
    }
    return on == 1;
}

int gemm_prepare(const WDesc& w, GemmPlan& plan, cudaStream_t st, std::string& err) {
    plan = GemmPlan();
    if (!tc_enabled() || w.K >= 32768 || w.N <= 0 || w.K <= 0) return SLX_OK;
    // Factor each row's common trailing zero bits out of its composites (restored exactly in the
    // epilogue), so the digit planes hold fewer significant bits.
    if (cudaMalloc(&plan.row_shift, (size_t)w.N) != cudaSuccess) { err = "device allocation failed"; return SLX_EOOM; }
    tc::weight_tz(w, plan.row_shift, st);
    int maxd = tc::weight_digits(w, st, err, plan.row_shift);
    if (maxd < 0) return SLX_ECUDA;
    if (maxd > 4) {  // composites too wide for the digit path: exact kernel
        cudaFree(plan.row_shift);
        plan.row_shift = nullptr;
        return SLX_OK;
    }
    plan.wlimbs = maxd < 1 ? 1 : maxd;
    plan.n_pad = round_up(w.N, tc::BN);
    plan.k_pad = round_up(w.K, tc::BK);
    plan.limb_bytes = (size_t)plan.wlimbs * plan.n_pad * plan.k_pad;
    if (cudaMalloc(&plan.limbs, plan.limb_bytes) != cudaSuccess) { err = "device allocation failed"; return SLX_EOOM; }
    tc::split_w(w, plan.wlimbs, plan.n_pad, plan.k_pad, (int8_t*)plan.limbs, st, plan.row_shift);
    if (!tc::encode_planes(plan.tmap_w, plan.limbs, plan.k_pad, plan.n_pad, plan.wlimbs, tc::GN, 1, tc::GK)) {
        cudaFree(plan.limbs);
        cudaFree(plan.row_shift);
        plan = GemmPlan();
        return SLX_OK;  // no tensor-map encoder available: exact kernel
    }
    plan.use_tc = 1;
    return SLX_OK;
}

int gemm_run(const int64_t* a, int64_t lda, int M, const WDesc& w, const GemmPlan& plan, int64_t* c, int64_t ldc,
             int shift, const int64_t* r, int64_t ldr, GemmWorkspace& ws, cudaStream_t st) {
    if (M <= 0) return 0;
    if (!r && gemv_supported(w, M) && gemv_reserve(ws, M, (int)w.N, (int)w.K, st))  // decode-shaped: stream the packed blocks once
        return gemv_exact(a, lda, M, w, c, ldc, shift, ws, st);
    if (!plan.use_tc) return gemm_exact(a, lda, M, (int)w.K, w, c, ldc, shift, r, ldr, st);
    const int64_t mpad = round_up(M, tc::BM);
    const size_t need = (size_t)tc::LA * mpad * plan.k_pad + 256;
    if (need > ws.bytes) {
        if (ws.p) cudaFree(ws.p);
        ws.p = nullptr;
        ws.bytes = 0;
        ws.gen++;
        if (cudaMalloc(&ws.p, need) != cudaSuccess) return gemm_exact(a, lda, M, (int)w.K, w, c, ldc, shift, r, ldr, st);
        ws.bytes = need;
        cudaMemsetAsync(ws.p, 0, need, st);  // flag words, and the GEMV's row-tile counters start at zero
    }
    int* flag = (int*)ws.p;
    int8_t* planes = (int8_t*)ws.p + 256;
    alignas(64) unsigned char tmap_a[128];
    if (!tc::encode_planes(tmap_a, planes, plan.k_pad, mpad, tc::LA, tc::GM, 1, tc::GK))
        return gemm_exact(a, lda, M, (int)w.K, w, c, ldc, shift, r, ldr, st);
    cudaMemsetAsync(flag, 0, sizeof(int), st);
    tc::split_a(a, lda, M, (int)w.K, mpad, plan.k_pad, planes, flag, st);
    // (the exact product runs in the same launch if the split overflowed)
    tc::launch(tmap_a, plan.tmap_w, plan.wlimbs, M, (int)w.N, (int)w.K, mpad, plan.n_pad, plan.k_pad, shift, c, ldc, r,
               ldr, flag, ws.err, st, plan.row_shift, ws.wait, a, lda, &w);
    return 2;
}

int gemm_run_multi(const int64_t* a, int64_t lda, int M, int n, const WDesc* const* w, const GemmPlan* const* plan,
                   int64_t* const* c, const int64_t* ldc, int shift, GemmWorkspace& ws, cudaStream_t st) {
    if (M <= 0 || n <= 0) return 0;
    bool shared = true;
    for (int i = 0; i < n; i++)
        shared = shared && plan[i]->use_tc && plan[i]->k_pad == plan[0]->k_pad && w[i]->K == w[0]->K &&
                 !gemv_supported(*w[i], M);
    if (!shared) {
        int q = 0;
        for (int i = 0; i < n; i++) q += gemm_run(a, lda, M, *w[i], *plan[i], c[i], ldc[i], shift, nullptr, 0, ws, st);
        return q;
    }
    const int64_t mpad = round_up(M, tc::BM), kpad = plan[0]->k_pad;
    const size_t need = (size_t)tc::LA * mpad * kpad + 256;
    if (need > ws.bytes) {
        if (ws.p) cudaFree(ws.p);
        ws.p = nullptr;
        ws.bytes = 0;
        ws.gen++;
        if (cudaMalloc(&ws.p, need) != cudaSuccess) {
            int q = 0;
            for (int i = 0; i < n; i++) q += gemm_exact(a, lda, M, (int)w[i]->K, *w[i], c[i], ldc[i], shift, nullptr, 0, st);
            return q;
        }
        ws.bytes = need;
        cudaMemsetAsync(ws.p, 0, need, st);  // flag words, and the GEMV's row-tile counters start at zero
    }
    int* flag = (int*)ws.p;
    int8_t* planes = (int8_t*)ws.p + 256;
    alignas(64) unsigned char tmap_a[128];
    if (!tc::encode_planes(tmap_a, planes, kpad, mpad, tc::LA, tc::GM, 1, tc::GK)) {
        int q = 0;
        for (int i = 0; i < n; i++) q += gemm_exact(a, lda, M, (int)w[i]->K, *w[i], c[i], ldc[i], shift, nullptr, 0, st);
        return q;
    }
    cudaMemsetAsync(flag, 0, sizeof(int), st);
    tc::split_a(a, lda, M, (int)w[0]->K, mpad, kpad, planes, flag, st);
    for (int i = 0; i < n; i++) {
        tc::launch(tmap_a, plan[i]->tmap_w, plan[i]->wlimbs, M, (int)w[i]->N, (int)w[i]->K, mpad, plan[i]->n_pad, kpad,
                   shift, c[i], ldc[i], nullptr, 0, flag, ws.err, st, plan[i]->row_shift, ws.wait, a, lda, w[i]);
    }
    return 1 + n;
}

bool gemm_run_planes(const int8_t* planes, const int* flag, const int64_t* a, int64_t lda, int M, const WDesc& w,
                     const GemmPlan& plan, int64_t* c, int64_t ldc, int shift, const int64_t* r, int64_t ldr,
                     GemmWorkspace& ws, cudaStream_t st) {
    if (M <= 0 || !plan.use_tc || (!r && gemv_supported(w, M))) return false;
    const int64_t mpad = round_up(M, tc::BM);
    alignas(64) unsigned char tmap_a[128];
    if (!tc::encode_planes(tmap_a, const_cast<int8_t*>(planes), plan.k_pad, mpad, tc::LA, tc::GM, 1, tc::GK)) return false;
    // (the exact product runs in the same launch if a value overflowed its digits)
    tc::launch(tmap_a, plan.tmap_w, plan.wlimbs, M, (int)w.N, (int)w.K, mpad, plan.n_pad, plan.k_pad, shift, c, ldc, r,
               ldr, flag, ws.err, st, plan.row_shift, ws.wait, a, lda, &w);
    return true;
}

void gemm_workspace_free(GemmWorkspace& ws) {
    if (ws.p) cudaFree(ws.p);
    ws.p = nullptr;
    ws.bytes = 0;
}

}  // namespace slx
