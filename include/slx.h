/* slx.h -- C ABI of libslx, the sm_100a implementation of SparseLattice's quantized integer
 * transformer forward path (GGUF dequantization fused into the Q30 matrix products of the
 * nomic-bert encoder and the Gemma causal LM, with the integer attention, norms and FFN).
 *
 * Plain C types only; no CUDA or framework types in the signatures. Every entry point returns an
 * slx_status; a message for the last failure on a context is available from slx_last_error().
 * Host-buffer entry points copy in and out and return when the result is on the host. Device
 * entry points (suffix _device) take device pointers and a stream handle (cudaStream_t passed as
 * void*, NULL = the context's stream) and return once the work is queued.
 *
 * Citations are to the reference project damiant3/SpatialDb, directory SparseLattice/.
 */
#ifndef SLX_H
#define SLX_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. The C# shim maps them back to the reference's exception types. */
typedef int slx_status;
#define SLX_OK 0
#define SLX_EINVAL 1        /* ArgumentException: bad shape, null pointer, bad kind */
#define SLX_EFORMAT 2       /* InvalidDataException: bad magic / version / value type */
#define SLX_ENOTFOUND 3     /* FileNotFoundException / KeyNotFoundException */
#define SLX_EUNSUPPORTED 4  /* NotSupportedException: dtype or architecture */
#define SLX_EEOF 5          /* EndOfStreamException: truncated tensor data */
#define SLX_ERANGE 6        /* IndexOutOfRangeException: MXFP4 nibble 15, RoPE row past its table */
#define SLX_EOOM 7          /* device allocation failed */
#define SLX_ECUDA 8         /* CUDA runtime error */
#define SLX_ETIMEOUT 9      /* a bounded device wait gave up */
#define SLX_ESCRATCH 10     /* the request is larger than slx_matmul_q30_noalloc's fixed scratch */

/* Model kinds for slx_model_load_gguf. */
#define SLX_MODEL_ENCODER 0       /* IntegerTransformerSource (nomic-bert / bert) */
#define SLX_MODEL_CAUSAL 1        /* IntegerCausalSource (gemma*) */
#define SLX_MODEL_GEMMA_ENCODER 2 /* IntegerGemmaSource (gemma*, non-causal, mean pooled) */
#define SLX_MODEL_FLOAT_ENCODER 3 /* TransformerEmbeddingSource (nomic-bert / bert), the fp32 twin: slx_encode
                                     fills l2 only (pooled_q30 must be NULL); agrees with the reference to
                                     fp32 rounding (SIMD dot order), not bit for bit */

typedef struct slx_ctx slx_ctx;
typedef struct slx_model slx_model;

/* ---- context ------------------------------------------------------------------------------ */
/* Binds a CUDA device and creates the context's stream. No reference counterpart: the C# host
 * creates one context per thread or serialises calls on one. */
slx_status slx_init(int device, slx_ctx** out);
slx_status slx_destroy(slx_ctx* ctx);
/* Message of the last failure on ctx (valid until the next call on ctx). */
const char* slx_last_error(slx_ctx* ctx);
/* Library version string. */
const char* slx_version(void);
/* No reference counterpart (the reference's errors are exceptions thrown on the calling thread).
 * Device-side errors of work queued on ctx through the _device entry points -- a token id whose UNK
 * row is outside the table (SLX_ERANGE), a tensor-core GEMM that gave up on a bounded wait
 * (SLX_ETIMEOUT) -- are recorded in the context's error word, which stays set until it is read:
 * slx_ctx_status waits for `stream` (NULL = the context's stream), returns the recorded status and
 * clears it. The host-buffer entry points clear the word when they start and check it (reporting
 * and clearing what they find) before they return. */
slx_status slx_ctx_status(slx_ctx* ctx, void* stream);
/* Context options (no reference counterpart). SLX_OPT_WAIT_LIMIT_CYCLES: SM clock cycles after
 * which a wait inside the tensor-core projection GEMM gives up (0 = the default, about two seconds);
 * the kernel then lets its copies and MMAs in flight finish, frees its tensor memory, returns and
 * reports SLX_ETIMEOUT, leaving the context usable. SLX_OPT_TEST_STALL_MMA (testing only): nonzero
 * makes that GEMM's MMA warp issue nothing, so its pipeline waits run out and the timeout path runs
 * without any fault; results of such calls are undefined. */
#define SLX_OPT_WAIT_LIMIT_CYCLES 1
#define SLX_OPT_TEST_STALL_MMA 2
slx_status slx_ctx_set_option(slx_ctx* ctx, int option, int64_t value);

/* ---- GGUF ---------------------------------------------------------------------------------- */
/* GgufReader.ReadTensorF32 (Gguf/GgufReader.cs:141-145, 172-201) for one tensor of a file:
 * dequantizes on the device with GgufDequantizer's formulas and element orders
 * (Gguf/GgufDequantizer.cs:7-325) and copies `n` floats to host `out` (n = element count). */
slx_status slx_gguf_read_f32(slx_ctx* ctx, const char* path, const char* tensor, float* out, int64_t n);

/* GgufDequantizer.Dequantize* over raw block bytes already in host memory
 * (Gguf/GgufDequantizer.cs:19-325; dtype ids from Gguf/GgufTypes.cs:21-38). */
slx_status slx_dequantize(slx_ctx* ctx, int dtype, const uint8_t* raw, int64_t nbytes, float* out, int64_t n);

/* ---- models -------------------------------------------------------------------------------- */
/* IntegerTransformerSource.Load (Gguf/IntegerTransformerSource.Loading.cs:47-58),
 * IntegerCausalSource.Load (Gguf/IntegerCausalSource.Loading.cs:41-52) and
 * IntegerGemmaSource.Load (Gguf/IntegerGemmaSource.Loading.cs:58-69): parses the GGUF file and
 * uploads the packed weight blocks to device memory. scale_bits is the Q scale (30). */
slx_status slx_model_load_gguf(slx_ctx* ctx, const char* path, int kind, int scale_bits, slx_model** out);
slx_status slx_model_free(slx_model* model);
/* info[0..11]: kind, embd, heads, kv_heads, head_dim, ff, layers, vocab, eos, unk, q_dim, kv_dim. */
slx_status slx_model_info(slx_model* model, int32_t* info, int n);

/* ---- encoder (IEmbeddingSource, Embedding/IEmbeddingSource.cs:13-33) ----------------------- */
/* IntegerTransformerSource.Forward on token ids (Gguf/IntegerTransformerSource.cs:65-78) for B
 * sequences of T tokens each (EmbedBatchAsync's loop, :40-47, done as one batch): writes the
 * mean-pooled Q30 vectors pooled_q30[B][embd]. If l2 is not NULL it also receives ForwardFloat's
 * L2-normalised float vectors (:52-62, .Forward.cs:89-99). Also serves SLX_MODEL_GEMMA_ENCODER
 * (IntegerGemmaSource.Forward, Gguf/IntegerGemmaSource.cs:66-80). */
slx_status slx_encode(slx_model* model, const int32_t* ids, int B, int T, int64_t* pooled_q30, float* l2);
/* Same on device buffers: d_ids[B*T] int32, d_pooled[B*embd] int64, queued on `stream`. Errors the
 * device raises while it runs (SLX_ERANGE, SLX_ETIMEOUT) are read with slx_ctx_status. From the
 * second call of a (B, T) on, the integer encoder's forward is replayed from a CUDA graph the model
 * captured (same results; the graph's input and output live in the model's workspace, so d_ids and
 * d_pooled may change between calls). The replay is skipped, and the forward queued kernel by
 * kernel, while profiling, on the legacy default stream, while `stream` is itself being captured,
 * and for fewer than 64 rows. */
slx_status slx_encode_device(slx_model* model, const int32_t* d_ids, int B, int T, int64_t* d_pooled, void* stream);

/* Hidden states after the first n_layers blocks (n_layers < 0: all), x_q30[T][embd], for one
 * sequence: the state ForwardCausalWithTrace samples (Gguf/IntegerCausalSource.Forward.cs:154-176)
 * and the encoder equivalent; used to bisect parity by layer. final_norm applies the causal
 * model's output RmsNorm after the last block. */
slx_status slx_trace_hidden(slx_model* model, const int32_t* ids, int T, int n_layers, int final_norm, int64_t* x_q30);

/* ---- causal LM (IntegerCausalSource, Gguf/IntegerCausalSource.cs:86-200) ------------------- */
/* ForwardCausal (:128-147): last position's hidden state after the output norm, Q30. */
slx_status slx_causal_forward_last(slx_model* model, const int32_t* ids, int T, int64_t* last_q30);
/* ForwardCausalFloat + PredictNextToken without lattice (:114-122, :149-161): greedy next id
 * from VocabLattice.ArgmaxBruteForce (Lattice/VocabLattice.cs:103-126), for B sequences of T. */
slx_status slx_causal_next_token(slx_model* model, const int32_t* ids, int B, int T, int32_t* next);
/* Generate on token ids (:86-108): full re-forward per step, greedy, stops at EOS (not
 * emitted). B independent prompts of T tokens; out[B][max_new] receives the new ids and
 * n_out[B] their counts. */
slx_status slx_causal_generate(slx_model* model, const int32_t* ids, int B, int T, int max_new, int32_t* out,
                               int32_t* n_out);
/* PredictNextToken with the VocabLattice (:149-157, Lattice/VocabLattice.cs:15-76): the rows of
 * TokenEmbeddingsFloat ((float)Half, :51-62) and the float hidden state are quantized with
 * ZeroThreshold 0.001 and GlobalScale 1e9; the k rows nearest by DistanceSquaredL2Fast
 * (Math/SparseVector.cs:138-169) are scored by their sequential fp32 dot with the hidden state and
 * the highest score wins. Ties have no defined order in the reference (unstable sorts): equal
 * distances go by ascending row, equal scores to the nearer candidate. k <= 0 (no candidate) gives
 * EOS; k > 8192 is SLX_EINVAL. The lattice is built on the device at the first call. */
slx_status slx_causal_next_token_lattice(slx_model* model, const int32_t* ids, int B, int T, int k, int32_t* next);
/* Generate(useLattice: true, latticeK: k) on token ids (:86-108), B prompts as slx_causal_generate. */
slx_status slx_causal_generate_lattice(slx_model* model, const int32_t* ids, int B, int T, int max_new, int k,
                                       int32_t* out, int32_t* n_out);
/* VocabLattice.QueryTopK (Lattice/VocabLattice.cs:43-58) of a causal model's lattice for B float
 * hidden states [B][embd]: ids[B][k] ascending by (distance, row), -1 past the vocabulary; dist
 * (nullable) [B][k] their DistanceSquaredL2Fast values, UINT64_MAX past the vocabulary. */
slx_status slx_vocab_lattice_query(slx_model* model, const float* hidden, int B, int k, int32_t* ids, uint64_t* dist);

/* ---- kernel-level ---------------------------------------------------------------------------- */
/* IntegerMatMul.MatMul with GGUF weights (Math/IntegerMatMul.cs:37-76 for the long composite,
 * :166-205 for the Half composite): c[M][N] = (long)((sum_k a[M][K] * w[n][k]) >> shift), where
 * w is the Q30 composite of the GGUF tensor `w_raw` (dtype, N rows of K, flat block order) formed
 * as IntegerTransformerSource (half_composite = 0) or IntegerCausalSource (half_composite = 1)
 * forms it. Host buffers. */
slx_status slx_matmul_q30(slx_ctx* ctx, const int64_t* a, int M, int K, int dtype, const uint8_t* w_raw,
                          int64_t w_bytes, int N, int half_composite, int scale_bits, int shift, int64_t* c);
/* Same on device buffers (a, w_raw, c device pointers), queued on `stream`. Decode-shaped calls
 * (M <= 8, Q4_0 / Q8_0, long composite, K a multiple of 32) stream the packed blocks and return
 * once queued; other shapes build the weight's tensor-core digit planes for the call and return
 * after the stream has finished with them. */
slx_status slx_matmul_q30_device(slx_ctx* ctx, const int64_t* d_a, int M, int K, int dtype, const uint8_t* d_w,
                                 int64_t w_bytes, int N, int half_composite, int scale_bits, int shift, int64_t* d_c,
                                 void* stream);

/* IntegerMatMul.MatMul with a weight prepared once (Math/IntegerMatMul.cs:37-76 / :166-205), the way
 * the model sources use their weights: the reference converts every weight at load
 * (Gguf/IntegerTransformerSource.Loading.cs:105-119 to Q30 long[], Gguf/IntegerCausalSource.Loading.cs:218-225
 * to Half[]) and multiplies many activations by it. slx_weight_prepare builds the tensor-core digit
 * planes of the composites of the GGUF blocks at d_w (device memory the caller keeps alive while the
 * handle lives) and waits for them; slx_matmul_q30_prepared queues c[M][N] = MatMul(d_a[M][K], w) >>
 * shift on `stream` (M <= 8 with Q4_0 / Q8_0 and the long composite streams the packed blocks
 * instead). info: N, K, tensor-core path (1) or exact kernel (0), weight digits. */
typedef struct slx_weight slx_weight;
slx_status slx_weight_prepare(slx_ctx* ctx, const uint8_t* d_w, int64_t w_bytes, int dtype, int N, int K,
                              int half_composite, int scale_bits, slx_weight** out);
slx_status slx_weight_free(slx_weight* w);
slx_status slx_weight_info(slx_weight* w, int32_t* info, int n);
slx_status slx_matmul_q30_prepared(slx_weight* w, const int64_t* d_a, int M, int shift, int64_t* d_c, void* stream);

/* No counterpart in the reference: slx_matmul_q30_device for callers that must not allocate device
 * memory -- services whose GPU memory is owned by another allocator (a framework's caching
 * allocator or a pre-sized arena), where a cudaMalloc inside a request fails or breaks the budget,
 * and latency-bound request paths that cannot pay for cudaMalloc and its implicit device
 * synchronisation. Same arguments and bit-exact result as slx_matmul_q30_device (ldc = N), on the
 * current CUDA device, but every intermediate lives in a fixed scratch array compiled into the
 * library (SLX_NOALLOC_SCRATCH_BYTES on every device that loads it, held until exit).
 * Limit: 256 + 5*ceil(M/128)*128*ceil(K/128)*128 + 4*ceil(N/64)*64*ceil(K/128)*128 bytes must fit
 * the scratch and K < 32768, else SLX_ESCRATCH. The first call on a device looks up the scratch
 * address there (cudaGetSymbolAddress) and keeps it for the life of the process, so the entry point
 * must not be used on a device after a cudaDeviceReset (or primary-context reset) there. The call is
 * synchronous: it reads the call's error word back and waits for its work on `stream` to finish
 * before it returns, so it cannot be captured into a CUDA graph. All calls share the scratch: calls
 * whose GPU work overlaps (other streams or threads on the same device) race and must be serialised. */
#define SLX_NOALLOC_SCRATCH_BYTES (32u << 20)
slx_status slx_matmul_q30_noalloc(const int64_t* d_a, int M, int K, int dtype, const uint8_t* d_w, int64_t w_bytes,
                                  int N, int half_composite, int scale_bits, int shift, int64_t* d_c, void* stream);

/* IntegerAttention on Q30 host arrays for one sequence (Math/IntegerAttention.cs):
 * mode 0 MultiHeadAttention / GroupedQueryAttention (:60-109, :125-202), mode 1
 * CausalGroupedQueryAttention (:205-289, leaky -2^29 mask), mode 2 SlidingWindowCausalGQA
 * (:293-377). q[seq][q_embd], k and v [seq][kv_dim], out[seq][q_embd]; scale_exp as the
 * reference's scaleExponent (score shift 2|scale_exp| - 30). */
slx_status slx_attention(slx_ctx* ctx, const int64_t* q, const int64_t* k, const int64_t* v, int seq, int q_embd,
                         int kv_dim, int n_heads, int n_kv_heads, int scale_exp, int mode, int window, int64_t* out);

/* ---- lattice k-NN search ------------------------------------------------------------------------ */
/* The embed+search path: EmbeddingLattice<TPayload>(occupants) + QueryKNearestL2(center, k)
 * (Lattice/EmbeddingLattice.cs:70-77) over vectors quantized by EmbeddingAdapter.Quantize
 * (Math/EmbeddingAdapter.cs:15-41), as VocabLattice builds and queries it (Lattice/VocabLattice.cs:15-58):
 * rows are float embeddings, quantized with (zero_threshold, global_scale) -- VocabLattice uses
 * 0.001 and 1e9 -- and every query is quantized with the lattice's options. The answer is exact:
 * the k smallest SparseVector.DistanceSquaredL2Fast distances (Math/SparseVector.cs:138-169),
 * ascending; equal distances are ordered by id (the reference leaves them to an unstable sort).
 * ids are id_base + row (so shards of one database can carry global ids); entries past the
 * database are id -1 with distance UINT64_MAX (the reference returns a shorter list). A quantized
 * component outside int32 is SLX_ERANGE; dim <= 16384; 0 <= k <= 16. */
typedef struct slx_lattice slx_lattice;
#define SLX_KNN_EXACT 1 /* query flag: skip the tensor-core bound, scan every row exactly */
slx_status slx_lattice_build(slx_ctx* ctx, const float* vectors, int64_t n, int dim, float zero_threshold,
                             int64_t global_scale, int64_t id_base, slx_lattice** out);
slx_status slx_lattice_build_device(slx_ctx* ctx, const float* d_vectors, int64_t n, int dim, float zero_threshold,
                                    int64_t global_scale, int64_t id_base, void* stream, slx_lattice** out);
slx_status slx_lattice_free(slx_lattice* lat);
/* info: n rows, dim, id_base */
slx_status slx_lattice_info(slx_lattice* lat, int64_t* info, int n);
/* ids [nq][k], dist [nq][k]; n_exact (nullable) = queries the bound could not decide, answered by an
 * exact scan. The device variant synchronizes its stream once (to size that scan). */
slx_status slx_lattice_query_knn_l2(slx_lattice* lat, const float* queries, int nq, int k, int flags, int64_t* ids,
                                    uint64_t* dist, int* n_exact);
slx_status slx_lattice_query_knn_l2_device(slx_lattice* lat, const float* d_queries, int nq, int k, int flags,
                                           int64_t* d_ids, uint64_t* d_dist, int* n_exact, void* stream);
/* KD tree over a lattice's rows: EmbeddingLatticeBuilder.Build (Lattice/EmbeddingLatticeBuilder.cs:11-127)
 * with LatticeOptions.LeafThreshold, as the EmbeddingLattice constructor runs it (row i is occupant i).
 * Spans of more than leaf_threshold occupants split at the median (sorted[N/2]) of their
 * highest-variance dimension, partitioned by the reference's two-pointer swap, so leaves hold the
 * reference's occupants in the reference's order. Equal variances take the lowest dimension (the
 * reference's ConcurrentDictionary enumeration order is machine-dependent). Built on the device. */
slx_status slx_lattice_build_tree(slx_lattice* lat, int leaf_threshold);
/* SparseTreeStats (EmbeddingLattice.CollectStats, Lattice/EmbeddingLattice.cs:102-150):
 * info = {TotalNodes, BranchNodes, LeafNodes, TotalOccupants, MaxDepth}. */
slx_status slx_lattice_tree_info(slx_lattice* lat, int64_t* info, int n);
/* The tree in pre-order (the serializer's order), TotalNodes entries per array (each nullable):
 * kind 0 leaf / 1 branch, child mask (1 below, 2 above), split dimension and value, and for leaves
 * the start and count of their occupants in perm (row index of every leaf-order position). */
slx_status slx_lattice_tree_export(slx_lattice* lat, int32_t* kind, int32_t* mask, int32_t* dim, int64_t* val,
                                   int64_t* start, int64_t* count, int32_t* perm);
/* SparseLatticeSerializer.Save with Int32PayloadSerializer (Lattice/SparseLatticeSerializer.cs:27-114):
 * the tree's SLAT bytes, payload = id_base + row (or the payloads a loaded lattice carries).
 * SLX_EINVAL without a tree (InvalidOperationException "must be frozen"). The _mem variant writes
 * to out (cap bytes; out may be NULL to query *size). */
slx_status slx_lattice_save_slat(slx_lattice* lat, const char* path);
slx_status slx_lattice_save_slat_mem(slx_lattice* lat, uint8_t* out, int64_t cap, int64_t* size);
/* SparseLatticeSerializer.Load with Int32PayloadSerializer (:46-166): a lattice whose rows are the
 * file's occupants in file order, with their tree; query ids are the payloads; queries are quantized
 * with (zero_threshold, global_scale). Errors: bad magic / version / tag SLX_EFORMAT, short input
 * SLX_EEOF, invalid occupants (SparseVector's checks) SLX_EINVAL, components beyond int32 SLX_ERANGE,
 * occupants of different widths or wider than 16384 SLX_EUNSUPPORTED, missing file SLX_ENOTFOUND. */
slx_status slx_lattice_load_slat(slx_ctx* ctx, const char* path, float zero_threshold, int64_t global_scale,
                                 slx_lattice** out);
slx_status slx_lattice_load_slat_mem(slx_ctx* ctx, const uint8_t* bytes, int64_t n, float zero_threshold,
                                     int64_t global_scale, slx_lattice** out);
/* k-way merge of per-shard answers: d_ids/d_dist [parts][nq][k] (each list ascending, as returned
 * above) -> [nq][k]; parts <= 64. No reference counterpart: the sharded database's top-k merge after
 * an all-gather of the shards' answers. */
slx_status slx_knn_merge_device(slx_ctx* ctx, const int64_t* d_ids, const uint64_t* d_dist, int parts, int nq, int k,
                                int64_t* d_out_ids, uint64_t* d_out_dist, void* stream);

/* ---- measurement ---------------------------------------------------------------------------- */
/* No reference counterpart (the reference times with Stopwatch, SparseLattice.Perf/Program.cs:817-830).
 * Per kernel class, the library's launches on ctx between begin and end, their device time from
 * CUDA events recorded on the launch stream, the algorithmic multiply-accumulates they performed
 * and, for the tensor-core projections, the int8 digit products issued. Classes: gemm, attention, norm, rope, ffn_gate, embed, pool, add, argmax, gemv, split, fallback,
 * search, vocab. */
typedef struct slx_kernel_stat {
    char name[24];
    int64_t launches;
    double ms;
    double macs;
    double bytes;
    double tc_macs;  /* int8 multiply-accumulates issued on the tensor cores (digit products) */
} slx_kernel_stat;
slx_status slx_profile_begin(slx_ctx* ctx);
slx_status slx_profile_end(slx_ctx* ctx, slx_kernel_stat* stats, int cap, int* n);
/* Running count of kernels the library has queued on ctx. */
slx_status slx_launch_count(slx_ctx* ctx, int64_t* launches);

#ifdef __cplusplus
}
#endif
#endif /* SLX_H */
