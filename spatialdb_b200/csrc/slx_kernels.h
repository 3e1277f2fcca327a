// slx_kernels.h -- launchers for the slx device kernels (host-callable, stream-ordered).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace slx {

// A GGUF weight tensor resident in device memory, addressed in the reference's flat element order
// (element e of row n is n*K + k; 32-element blocks run across row ends exactly as
// GgufDequantizer decodes a whole tensor). dtype is one of the natively decoded block formats
// (F32, F16, BF16, Q8_0, Q4_0); other GGUF formats are expanded to F32 at load.
struct WDesc {
    int dtype = 0;
    const uint8_t* data = nullptr;
    int64_t nblocks = 0;   // 32-element blocks present (Q8_0 / Q4_0)
    int64_t elements = 0;  // N*K
    int64_t N = 0, K = 0;
    int mode = 0;          // composite: 0 = (long)(f*2^s), 1 = (long)((float)(Half)f*2^s)
    double scale = 1073741824.0;
};

// Device-side error flags set by kernels instead of trapping (read back by the host).
enum : int { KERR_NONE = 0, KERR_RANGE = 1, KERR_TIMEOUT = 2 };

// c[M][N] = lo64((sum_k a[m][k] * w[n][k]) >> shift) (+ r[m][n] if r), exact Int128 accumulation.
// With only_if, the kernel does nothing unless *only_if is nonzero (device-side gate).
int gemm_exact(const int64_t* a, int64_t lda, int M, int K, const WDesc& w, int64_t* c, int64_t ldc, int shift,
                const int64_t* r, int64_t ldr, cudaStream_t st, const int* only_if = nullptr);

// Q30 composite of elements [0, n) of a weight into out (norm vectors, token-type rows).
int weight_to_q30(const WDesc& w, int64_t n, int64_t* out, cudaStream_t st);

// Any decodable GGUF dtype -> float (GgufDequantizer.cs formulas), n elements; sets *flag on an
// MXFP4 nibble 15 (the reference's IndexOutOfRangeException).
int dequant_f32(int dtype, const uint8_t* raw, int64_t n, float* out, int* flag, cudaStream_t st);

// x[b*T+t][j] = Q30(tok[id]) + tt[j]   (IntegerTransformerSource.BuildEmbeddings)
int embed_encoder(const int32_t* ids, int B, int T, const WDesc& tok, const int64_t* tt, int unk, int64_t* x,
                   int* flag, cudaStream_t st);
// x = Q30((Half)tok[id]) * sqrt_d  (IntegerCausalSource.BuildEmbeddings); long rows when tok_q30 mode 0
int embed_scaled(const int32_t* ids, int B, int T, const WDesc& tok, int unk, int64_t sqrt_d, int64_t* x, int* flag,
                  cudaStream_t st);

// LayerNorm rows (IntegerLayerNorm.NormalizeRow): rows of length n at x + r*ld.
int layernorm_rows(int64_t* x, int64_t ld, int rows, int n, const int64_t* w, const int64_t* b, cudaStream_t st);
// The same LayerNorm (n % 4 == 0, 16-byte aligned rows) with, when planes is not null, the outputs'
// digit planes [5][Mpad][Kpad] written alongside (the next projection's operand, zero padded) and
// *overflow raised for a value beyond five digits. Returns -1 (nothing queued) for shapes it does
// not cover.
int layernorm_rows_digits(int64_t* x, int64_t ld, int rows, int n, const int64_t* w, const int64_t* b, int64_t Mpad,
                          int64_t Kpad, int8_t* planes, int* overflow, cudaStream_t st);
// RmsNorm rows (IntegerLayerNorm.RmsNormRow): row r is segment (r % per) of line (r / per),
// x + (r/per)*ld + (r%per)*n, length n; per > 1 gives RmsNormPerHead.
int rmsnorm_rows(int64_t* x, int64_t ld, int rows, int per, int n, const int64_t* w, cudaStream_t st);
// The causal block's norm pair over rows of n (contiguous, n a multiple of 1024, at most 4096):
// with w1, y = RmsNormRow(y; w1) + r; with w2, z = RmsNormRow(y; w2), plus z's five digit planes
// [5][Mpad][Kpad = n] when planes is given (*overflow raised beyond five digits). Returns -1
// (nothing queued) for shapes it does not cover.
int rms_pair_rows(int64_t* y, const int64_t* r, int64_t* z, int rows, int n, const int64_t* w1, const int64_t* w2,
                  int64_t Mpad, int64_t Kpad, int8_t* planes, int* overflow, cudaStream_t st);

// ApplyRoPE on rows m of B*T (position m % T), nh heads of hd at x + m*ld + h*hd.
int rope_rows(int64_t* x, int64_t ld, int B, int T, int nh, int hd, const int64_t* cos, const int64_t* sin,
              cudaStream_t st, const int* only_if = nullptr);

// Attention for B sequences of T: q (ldq, nh heads of hd), k/v (ldk/ldv, nkv heads), out (ldo).
// mode 0 non-causal, 1 causal with the -2^(frac-1) mask, 2 sliding window.
// With only_if, the kernel does nothing unless *only_if is nonzero.
int attention(const int64_t* q, int64_t ldq, const int64_t* k, int64_t ldk, const int64_t* v, int64_t ldv,
               int64_t* out, int64_t ldo, int B, int T, int nh, int nkv, int hd, int score_shift, int64_t sqrt_hd,
               int mode, int window, cudaStream_t st, const int* only_if = nullptr);



// Same attention with tensor-core scores (k_attn.cu): digit split of q/k (with rope_cs / rope_sn
// given, ApplyRoPE is applied by the same pass to the values it splits; q and k themselves are
// rotated in place only when the exact kernel has to run, so afterwards they hold unspecified
// rotated or unrotated values), tcgen05 score GEMM,
// CUDA-core softmax and per-term PV, and the exact kernel gated behind them for out-of-range
// inputs. ws must hold attention_tc_workspace() bytes. Returns the kernels queued, -1 if the
// tensor maps could not be encoded (nothing queued). With planes (and kpad == nh * hd, mpad >= B * T)
// the P.V also writes the output rows' five activation digit planes [5][mpad][kpad] for the next
// projection; they are valid only while the int word at ws (attention_tc_flag) stays zero, which
// the caller passes to the projection as its fallback flag. Rows B*T..mpad are the caller's.
size_t attention_tc_workspace(int B, int T, int nh, int nkv, int hd);
bool attention_tc_supported(int T, int nh, int nkv, int hd);
int attention_tc(const int64_t* q, int64_t ldq, const int64_t* k, int64_t ldk, const int64_t* v, int64_t ldv,
                 int64_t* out, int64_t ldo, int B, int T, int nh, int nkv, int hd, int score_shift, int64_t sqrt_hd,
                 int mode, int window, void* ws, int* err, cudaStream_t st, const int64_t* rope_cs = nullptr,
                 const int64_t* rope_sn = nullptr, int8_t* planes = nullptr, int64_t mpad = 0, int64_t kpad = 0);
// The call's fallback flag inside ws: nonzero when the exact kernel produced the output.
inline const int* attention_tc_flag(const void* ws) { return (const int*)ws; }

// up[i] = (FixedSiLU(gate[i]) * up[i]) >> 30 over M rows of F (IntegerFFN)
int silu_gate(const int64_t* gate, int64_t ldg, int64_t* up, int64_t ldu, int M, int F, cudaStream_t st);
// The same gate, also writing the gated values' digit planes [5][Mpad][Kpad] (the next projection's
// operand, zero padded) and raising *overflow for a value beyond five digits. F % 4 == 0, rows 16-byte
// aligned (ldg, ldu even).
int silu_gate_digits(const int64_t* gate, int64_t ldg, int64_t* up, int64_t ldu, int M, int F, int64_t Mpad, int64_t Kpad,
                     int8_t* planes, int* overflow, cudaStream_t st);
// dst = dst + src (unchecked long adds) over M rows of n
int add_rows(int64_t* dst, int64_t ldd, const int64_t* src, int64_t lds, int M, int n, cudaStream_t st);
// pooled[b][j] = (long)(sum_t x[b*T+t][j] / T)  (MeanPool)
int mean_pool(const int64_t* x, int64_t ld, int B, int T, int d, int64_t* pooled, cudaStream_t st);
// Gather rows: dst[b] = src[b*T + T-1]
int gather_last_rows(const int64_t* x, int64_t ld, int B, int T, int d, int64_t* dst, cudaStream_t st);
// Greedy head: per sequence b, argmax over vocab rows of tok of sum_j h[j]*(float)(Half)tok[v][j]
// with h = (float)(last[b][j] * 2^-scale_bits), sequential fp32, first maximum wins.
int argmax_vocab(const int64_t* last, int B, int d, const WDesc& tok, int vocab, int scale_bits,
                  unsigned long long* keys, int32_t* ids, cudaStream_t st);

}  // namespace slx
