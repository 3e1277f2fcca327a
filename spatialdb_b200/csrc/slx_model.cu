// slx_model.cu -- model loading, forward orchestration and the extern "C" entry points of libslx.
//
// The forward passes restate, stage by stage, the reference sources:
//   encoder:  IntegerTransformerSource.Forward (Gguf/IntegerTransformerSource.cs:65-78) and
//             ApplyTransformerBlock (Gguf/IntegerTransformerSource.Forward.cs:28-67);
//   causal:   IntegerCausalSource.ForwardCausal (Gguf/IntegerCausalSource.cs:128-147) and
//             ApplyCausalBlock (Gguf/IntegerCausalSource.Forward.cs:45-114);
//   gemma encoder: IntegerGemmaSource.Forward (Gguf/IntegerGemmaSource.cs:66-80) and
//             ApplyGemmaBlock (Gguf/IntegerGemmaSource.Forward.cs:32-75).
// B independent sequences of T tokens run as one batch: every projection is one GEMM over B*T
// rows, attention and pooling stay per sequence.
#include <atomic>
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "gguf.hpp"
#include "slx.h"
#include "slx_kernels.h"
#include "slx_gemm.h"
#include "slx_search.h"
#include "slx_tree.h"
#include "slx_vocab.h"
#include "slx_float.h"

using namespace slx;

// Kernel classes reported by slx_profile_end.
enum KClass { KC_GEMM, KC_ATTENTION, KC_NORM, KC_ROPE, KC_FFN_GATE, KC_EMBED, KC_POOL, KC_ADD, KC_ARGMAX, KC_GEMV,
              KC_SPLIT, KC_FALLBACK, KC_SEARCH, KC_VOCAB, KC_COUNT };
static const char* kKClassName[KC_COUNT] = {"gemm", "attention", "norm", "rope", "ffn_gate", "embed", "pool", "add",
                                            "argmax", "gemv", "split", "fallback", "search", "vocab"};

struct ProfRecord {
    int cls;
    int launches;
    cudaEvent_t a, b;
    double macs, bytes, tc_macs;
};

struct slx_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    std::string err;
    int* d_flag = nullptr;
    int64_t launches = 0;            // kernels queued by the library on this context
    bool prof = false;
    std::vector<ProfRecord> records;
    GemmWorkspace kws;               // scratch of the kernel-level matmul entry points
    WaitOptions wait;                // bounded-wait settings of the tensor-core GEMMs (slx_ctx_set_option)
    std::atomic<int> refs{1};        // slx_destroy's reference plus one per live model, weight and lattice
    std::vector<cudaEvent_t> event_pool;
    cudaEvent_t event() {
        if (!event_pool.empty()) { cudaEvent_t e = event_pool.back(); event_pool.pop_back(); return e; }
        cudaEvent_t e = nullptr;
        cudaEventCreate(&e);
        return e;
    }
};

// Runs one launcher (which returns how many kernels it queued), counting launches and, when
// profiling, bracketing it with events on the launch stream.
template <class F>
static inline void run_k(slx_ctx* c, int cls, double macs, double bytes, cudaStream_t st, F&& f, double tc_macs = 0) {
    if (!c->prof) {
        c->launches += f();
        return;
    }
    ProfRecord r{cls, 0, c->event(), c->event(), macs, bytes, tc_macs};
    cudaEventRecord(r.a, st);
    r.launches = f();
    cudaEventRecord(r.b, st);
    c->launches += r.launches;
    c->records.push_back(r);
}

namespace {

int set_err(slx_ctx* c, int code, const char* fmt, ...) {
    if (!c) return code;
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    c->err = buf;
    return code;
}

#define CK(call)                                                                                 \
    do {                                                                                         \
        cudaError_t e_ = (call);                                                                 \
        if (e_ != cudaSuccess)                                                                   \
            return set_err(ctx, e_ == cudaErrorMemoryAllocation ? SLX_EOOM : SLX_ECUDA, "%s: %s", \
                           #call, cudaGetErrorString(e_));                                      \
    } while (0)

struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
};

// Exact floor sqrt of a non-negative long (ISqrt64, Math/IntegerLayerNorm.cs:130-149).
int64_t isqrt64_host(int64_t v) {
    if (v <= 0) return 0;
    int64_t x = (int64_t)std::sqrt((double)v);
    if (x <= 0) x = 1;
    while (x > 0 && (__int128)x * x > v) x--;
    while ((__int128)(x + 1) * (x + 1) <= v) x++;
    return x;
}

// IntegerRoPECache (Math/IntegerAttention.cs:14-32): built on the host in double precision with
// the C library's pow/cos/sin, truncated to Q30.
void rope_table(int rows, int hd, float base, std::vector<int64_t>& cs, std::vector<int64_t>& sn) {
    int half = hd / 2;
    cs.assign((size_t)rows * half, 0);
    sn.assign((size_t)rows * half, 0);
    auto q30 = [](double v) -> int64_t {
        double s = v * (double)(1LL << 30);
        if (s >= -9223372036854775808.0 && s < 9223372036854775808.0) return (int64_t)s;
        return INT64_MIN;
    };
    for (int t = 0; t < rows; t++)
        for (int i = 0; i < half; i++) {
            double theta = std::pow((double)base, -2.0 * i / hd);
            double angle = t * theta;
            cs[(size_t)t * half + i] = q30(std::cos(angle));
            sn[(size_t)t * half + i] = q30(std::sin(angle));
        }
}

}  // namespace

struct slx_model {
    slx_ctx* ctx = nullptr;
    int kind = 0, scale_bits = 30;
    int embd = 0, heads = 0, kv_heads = 0, head_dim = 0, q_dim = 0, kv_dim = 0, ff = 0, layers = 0;
    int vocab = 0, unk = 0, eos = 0, sliding = 0, global_interval = 0, rope_rows = 0;
    float rope_base = 10000.0f, rope_base_global = 10000.0f;
    std::vector<void*> allocs;
    WDesc tok;
    int64_t *tt = nullptr, *enw = nullptr, *enb = nullptr, *out_norm = nullptr;
    struct Layer {
        WDesc qkv, o, gate, up, down, q, k, v;
        GemmPlan p_qkv, p_o, p_gate, p_up, p_down, p_q, p_k, p_v;
        int64_t *anw = nullptr, *anb = nullptr, *lnw = nullptr, *lnb = nullptr;
        int64_t *attn_norm = nullptr, *qn = nullptr, *kn = nullptr, *post_attn = nullptr, *ffn_norm = nullptr,
                *post_ffw = nullptr;
    };
    std::vector<Layer> L;
    int64_t *cos_l = nullptr, *sin_l = nullptr, *cos_g = nullptr, *sin_g = nullptr;
    std::map<std::string, DevBuf> ws;
    GemmWorkspace gws;
    vocab::Lattice vlat;             // VocabLattice of the causal head, built on first use
    bool vlat_ready = false;
    fenc::Model fm;                  // SLX_MODEL_FLOAT_ENCODER: fp32 weights (in allocs)
    fenc::Workspace fws;
    uint64_t buf_gen = 0;            // bumped whenever buf() reallocates
    // The encoder forward of one (B, T) captured as a CUDA graph (encode_device): replayed while no
    // buffer it reads or writes has been reallocated since the capture.
    struct EncoderGraph {
        cudaGraphExec_t exec = nullptr;
        int B = -1, T = -1;
        uint64_t gen = 0;
        long long wait_limit = 0;
        int stall = 0;
        int64_t launches = 0;
        int seen_B = -1, seen_T = -1;  // the last eager forward, and the generation after it
        uint64_t seen_gen = ~0ull;
        bool disabled = false;
    } eg;
    uint64_t gen() const { return buf_gen + gws.gen; }

    ~slx_model() {
        if (eg.exec) cudaGraphExecDestroy(eg.exec);
        vocab::release(vlat);
        fws.release();
        for (auto& kv : ws) cudaFree(kv.second.p);
        for (void* p : allocs) cudaFree(p);
        gemm_workspace_free(gws);
    }

    template <class T>
    T* buf(const char* name, size_t count) {
        DevBuf& b = ws[name];
        size_t need = count * sizeof(T);
        if (need > b.bytes) {
            if (b.p) cudaFree(b.p);
            b.p = nullptr;
            buf_gen++;
            // A generate loop asks for one more token row every step: grow by at least a quarter, so
            // the buffers (and cudaFree's device synchronisation) are not renewed at every step.
            const size_t grown = b.bytes ? std::max(need, b.bytes + b.bytes / 4) : need;
            b.bytes = 0;
            if (cudaMalloc(&b.p, grown) != cudaSuccess) {
                if (grown == need || cudaMalloc(&b.p, need) != cudaSuccess) return nullptr;
                b.bytes = need;
            } else {
                b.bytes = grown;
            }
        }
        return (T*)b.p;
    }
};

namespace {

struct Loader {
    slx_ctx* ctx;
    slx_model* m;
    GgufFile& g;

    int upload(const void* src, size_t bytes, void** dst) {
        CK(cudaMalloc(dst, bytes ? bytes : 1));
        m->allocs.push_back(*dst);
        if (bytes) CK(cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice));
        return SLX_OK;
    }

    // A tensor as a weight descriptor; natively decoded dtypes stay packed, the rest are
    // dequantized once on the device to F32 (the float the reference itself would produce).
    int weight(const std::string& name, int64_t K, int64_t N, int mode, WDesc& w, bool need_shape = true) {
        const GgufTensor* t = g.tensor(name);
        if (!t) return set_err(ctx, SLX_ENOTFOUND, "Tensor '%s' not found in GGUF file", name.c_str());
        std::vector<uint8_t> raw;
        std::string err;
        int st = g.read_raw(*t, raw, err);
        if (st) return set_err(ctx, st, "%s", err.c_str());
        if (need_shape && t->elements < K * N)
            return set_err(ctx, SLX_ERANGE, "tensor '%s' has %lld elements, the forward indexes %lld", name.c_str(),
                           (long long)t->elements, (long long)(K * N));
        void* d = nullptr;
        if ((st = upload(raw.data(), raw.size(), &d))) return st;
        w = WDesc();
        w.K = K;
        w.N = N;
        w.elements = t->elements;
        w.mode = mode;
        w.scale = std::ldexp(1.0, m->scale_bits);
        switch (t->dtype) {
            case GG_F32: case GG_F16: case GG_BF16: case GG_Q8_0: case GG_Q4_0:
                w.dtype = (int)t->dtype;
                w.data = (const uint8_t*)d;
                w.nblocks = t->elements / 32;
                return SLX_OK;
            default: {
                float* f = nullptr;
                CK(cudaMalloc(&f, sizeof(float) * std::max<int64_t>(t->elements, 1)));
                m->allocs.push_back(f);
                CK(cudaMemsetAsync(ctx->d_flag, 0, sizeof(int), ctx->stream));
                dequant_f32((int)t->dtype, (const uint8_t*)d, t->elements, f, ctx->d_flag, ctx->stream);
                int flag = 0;
                CK(cudaMemcpyAsync(&flag, ctx->d_flag, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
                CK(cudaStreamSynchronize(ctx->stream));
                if (flag) return set_err(ctx, SLX_ERANGE, "MXFP4 nibble 15 in '%s' (index outside the 15-entry table)", name.c_str());
                w.dtype = GG_F32;
                w.data = (const uint8_t*)f;
                w.nblocks = 0;
                return SLX_OK;
            }
        }
    }

    // A vector tensor's first n elements as Q30 long (IntegerMatMul.QuantizeFromFloat).
    int vec_q30(const std::string& name, int64_t n, int64_t** out) {
        WDesc w;
        int st = weight(name, n, 1, 0, w);
        if (st) return st;
        CK(cudaMalloc((void**)out, sizeof(int64_t) * std::max<int64_t>(n, 1)));
        m->allocs.push_back(*out);
        weight_to_q30(w, n, *out, ctx->stream);
        return SLX_OK;
    }

    // A tensor read as float (GgufReader.ReadTensorF32), dequantized on the device; at least n elements.
    int f32(const std::string& name, int64_t n, float** out, int64_t* elements = nullptr) {
        const GgufTensor* t = g.tensor(name);
        if (!t) return set_err(ctx, SLX_ENOTFOUND, "Tensor '%s' not found in GGUF file", name.c_str());
        if (t->elements < n)
            return set_err(ctx, SLX_ERANGE, "tensor '%s' has %lld elements, the forward indexes %lld", name.c_str(),
                           (long long)t->elements, (long long)n);
        std::vector<uint8_t> raw;
        std::string err;
        int st = g.read_raw(*t, raw, err);
        if (st) return set_err(ctx, st, "%s", err.c_str());
        void* d = nullptr;
        CK(cudaMalloc(&d, std::max<size_t>(raw.size(), 1)));
        CK(cudaMemcpy(d, raw.data(), raw.size(), cudaMemcpyHostToDevice));
        CK(cudaMalloc((void**)out, sizeof(float) * std::max<int64_t>(t->elements, 1)));
        m->allocs.push_back(*out);
        CK(cudaMemsetAsync(ctx->d_flag, 0, sizeof(int), ctx->stream));
        dequant_f32((int)t->dtype, (const uint8_t*)d, t->elements, *out, ctx->d_flag, ctx->stream);
        int flag = 0;
        CK(cudaMemcpyAsync(&flag, ctx->d_flag, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
        CK(cudaStreamSynchronize(ctx->stream));
        cudaFree(d);
        if (flag) return set_err(ctx, SLX_ERANGE, "MXFP4 nibble 15 in '%s' (index outside the 15-entry table)", name.c_str());
        if (elements) *elements = t->elements;
        return SLX_OK;
    }

    int ones(int64_t n, int64_t** out) {  // MakeOnesWeight (IntegerCausalSource.Loading.cs:227-233)
        std::vector<int64_t> h((size_t)n, 1LL << m->scale_bits);
        return upload(h.data(), h.size() * sizeof(int64_t), (void**)out);
    }

    int vec_or_ones(const std::string& name, int64_t n, int64_t** out) {
        return g.tensor(name) ? vec_q30(name, n, out) : ones(n, out);
    }

    int rope(int rows, int hd, float base, int64_t** cs, int64_t** sn) {
        std::vector<int64_t> c, s;
        rope_table(rows, hd, base, c, s);
        int st = upload(c.data(), c.size() * 8, (void**)cs);
        if (st) return st;
        return upload(s.data(), s.size() * 8, (void**)sn);
    }
};

int lower_eq(const std::string& a, const char* b) {
    std::string x = a;
    std::transform(x.begin(), x.end(), x.begin(), ::tolower);
    return x == b;
}

// IntegerTransformerSource.LoadFromReader (Gguf/IntegerTransformerSource.Loading.cs:72-151)
int load_encoder(slx_ctx* ctx, slx_model* m, GgufFile& g) {
    if (!lower_eq(g.arch, "nomic-bert") && !lower_eq(g.arch, "bert"))
        return set_err(ctx, SLX_EUNSUPPORTED, "Architecture '%s' is not supported. Only 'nomic-bert' and 'bert' are implemented.", g.arch.c_str());
    m->embd = g.embd; m->heads = g.heads; m->kv_heads = g.heads; m->layers = g.layers; m->ff = g.ff;
    if (m->embd <= 0 || m->heads <= 0 || m->embd % m->heads) return set_err(ctx, SLX_EINVAL, "bad encoder dimensions");
    m->head_dim = m->embd / m->heads; m->q_dim = m->embd; m->kv_dim = m->embd;
    m->rope_base = g.get_float(g.arch + ".rope.freq_base", 10000.0f);
    Loader ld{ctx, m, g};
    int d = m->embd, F = m->ff, st;
    const GgufTensor* te = g.tensor("token_embd.weight");
    if (!te) return set_err(ctx, SLX_ENOTFOUND, "Tensor 'token_embd.weight' not found in GGUF file");
    if ((st = ld.weight("token_embd.weight", d, te->elements / d, 0, m->tok))) return st;
    if ((st = ld.vec_q30("token_types.weight", d, &m->tt))) return st;
    if ((st = ld.vec_q30("token_embd_norm.weight", d, &m->enw))) return st;
    if ((st = ld.vec_q30("token_embd_norm.bias", d, &m->enb))) return st;
    m->L.resize(m->layers);
    for (int i = 0; i < m->layers; i++) {
        std::string p = "blk." + std::to_string(i);
        auto& l = m->L[i];
        if ((st = ld.weight(p + ".attn_qkv.weight", d, 3 * d, 0, l.qkv))) return st;
        if ((st = ld.weight(p + ".attn_output.weight", d, d, 0, l.o))) return st;
        if ((st = ld.vec_q30(p + ".attn_output_norm.weight", d, &l.anw))) return st;
        if ((st = ld.vec_q30(p + ".attn_output_norm.bias", d, &l.anb))) return st;
        if ((st = ld.weight(p + ".ffn_up.weight", d, F, 0, l.up))) return st;
        if ((st = ld.weight(p + ".ffn_gate.weight", d, F, 0, l.gate))) return st;
        if ((st = ld.weight(p + ".ffn_down.weight", F, d, 0, l.down))) return st;
        if ((st = ld.vec_q30(p + ".layer_output_norm.weight", d, &l.lnw))) return st;
        if ((st = ld.vec_q30(p + ".layer_output_norm.bias", d, &l.lnb))) return st;
    }
    // WordPieceTokenizer.FromGguf (Gguf/WordPieceTokenizer.cs:23-30) rejects an empty vocabulary.
    if (g.n_tokens == 0) return set_err(ctx, SLX_EINVAL, "GGUF file contains no tokenizer vocabulary");
    m->unk = g.unk; m->eos = g.eos; m->vocab = g.n_tokens;
    m->rope_rows = 512;  // s_ropeMaxSeqLen (IntegerTransformerSource.cs:27)
    return ld.rope(m->rope_rows, m->head_dim, m->rope_base, &m->cos_g, &m->sin_g);
}

// TransformerEmbeddingSource.Load / LoadFromReader (Gguf/TransformerEmbeddingSource.cs:46-57,506-557):
// every tensor read as float; the RopeCache (:227-252) with theta = (float)Pow(base, -2i/hd) and
// angle = t * theta in double, 512 rows.
int load_float_encoder(slx_ctx* ctx, slx_model* m, GgufFile& g) {
    if (!lower_eq(g.arch, "nomic-bert") && !lower_eq(g.arch, "bert"))
        return set_err(ctx, SLX_EUNSUPPORTED, "Architecture '%s' is not supported. Only 'nomic-bert' and 'bert' are implemented.", g.arch.c_str());
    m->embd = g.embd; m->heads = g.heads; m->kv_heads = g.heads; m->layers = g.layers; m->ff = g.ff;
    if (m->embd <= 0 || m->heads <= 0 || m->embd % m->heads) return set_err(ctx, SLX_EINVAL, "bad encoder dimensions");
    m->head_dim = m->embd / m->heads; m->q_dim = m->embd; m->kv_dim = m->embd;
    m->rope_base = g.get_float(g.arch + ".rope.freq_base", 10000.0f);
    Loader ld{ctx, m, g};
    const int d = m->embd, F = m->ff;
    fenc::Model& fm = m->fm;
    fm.d = d; fm.heads = m->heads; fm.ff = F;
    int st;
    float* p = nullptr;
    int64_t tok_el = 0;
    if ((st = ld.f32("token_embd.weight", d, &p, &tok_el))) return st;
    fm.tok = p;
    fm.tok_rows = tok_el / d;
    if ((st = ld.f32("token_types.weight", d, &p))) return st;
    fm.tt = p;
    if ((st = ld.f32("token_embd_norm.weight", d, &p))) return st;
    fm.enw = p;
    if ((st = ld.f32("token_embd_norm.bias", d, &p))) return st;
    fm.enb = p;
    fm.layers.resize(m->layers);
    for (int i = 0; i < m->layers; i++) {
        const std::string pre = "blk." + std::to_string(i);
        fenc::Layer& l = fm.layers[i];
        const struct { const char* name; int64_t n; const float** dst; } t[9] = {
            {".attn_qkv.weight", (int64_t)3 * d * d, &l.qkv}, {".attn_output.weight", (int64_t)d * d, &l.o},
            {".attn_output_norm.weight", d, &l.anw}, {".attn_output_norm.bias", d, &l.anb},
            {".ffn_up.weight", (int64_t)F * d, &l.up}, {".ffn_gate.weight", (int64_t)F * d, &l.gate},
            {".ffn_down.weight", (int64_t)d * F, &l.down}, {".layer_output_norm.weight", d, &l.lnw},
            {".layer_output_norm.bias", d, &l.lnb}};
        for (const auto& e : t) {
            if ((st = ld.f32(pre + e.name, e.n, &p))) return st;
            *e.dst = p;
        }
    }
    if (g.n_tokens == 0) return set_err(ctx, SLX_EINVAL, "GGUF file contains no tokenizer vocabulary");
    m->unk = g.unk; m->eos = g.eos; m->vocab = g.n_tokens;
    fm.unk = g.unk;
    m->rope_rows = 512;  // RopeMaxSeqLen (TransformerEmbeddingSource.cs:254)
    const int hd = m->head_dim, half = hd / 2;
    std::vector<float> cs((size_t)512 * std::max(half, 1)), sn(cs.size());
    for (int t2 = 0; t2 < 512; t2++)
        for (int i = 0; i < half; i++) {
            const float theta = (float)std::pow((double)m->rope_base, -2.0 * i / hd);
            const double angle = t2 * (double)theta;
            cs[(size_t)t2 * half + i] = (float)std::cos(angle);
            sn[(size_t)t2 * half + i] = (float)std::sin(angle);
        }
    void* dc = nullptr;
    void* ds = nullptr;
    if ((st = ld.upload(cs.data(), cs.size() * 4, &dc)) || (st = ld.upload(sn.data(), sn.size() * 4, &ds))) return st;
    fm.cos = (const float*)dc;
    fm.sin = (const float*)ds;
    m->fws.err = ctx->d_flag;
    if (tc_enabled()) {  // the projections' weights split once for the tensor-core path
        for (fenc::Layer& l : fm.layers) {
            const struct { const float* w; int N, K; const float** dst; } t[5] = {
                {l.qkv, 3 * d, d, &l.qkv_t}, {l.o, d, d, &l.o_t}, {l.up, F, d, &l.up_t}, {l.gate, F, d, &l.gate_t},
                {l.down, d, F, &l.down_t}};
            for (const auto& e : t) {
                void* pl = nullptr;
                CK(cudaMalloc(&pl, fenc::tc_weight_bytes(e.N, e.K)));
                m->allocs.push_back(pl);
                if (!fenc::tc_prepare_weight(e.w, e.N, e.K, (float*)pl, 0)) return set_err(ctx, SLX_ECUDA, "weight split failed");
                *e.dst = (const float*)pl;
            }
        }
        CK(cudaDeviceSynchronize());
    }
    return SLX_OK;  // m->L stays empty: no integer projections to plan
}

// IntegerCausalSource.LoadFromReader (Gguf/IntegerCausalSource.Loading.cs:74-195); with
// gemma_encoder, IntegerGemmaSource.LoadFromReader (Gguf/IntegerGemmaSource.Loading.cs:80-157).
int load_causal(slx_ctx* ctx, slx_model* m, GgufFile& g, bool gemma_encoder) {
    std::string a = g.arch, al = a;
    std::transform(al.begin(), al.end(), al.begin(), ::tolower);
    if (al.rfind("gemma", 0) != 0) return set_err(ctx, SLX_EUNSUPPORTED, "Architecture '%s' is not supported.", a.c_str());
    m->embd = g.embd; m->heads = g.heads; m->layers = g.layers; m->ff = g.ff;
    if (m->embd <= 0 || m->heads <= 0) return set_err(ctx, SLX_EINVAL, "bad model dimensions");
    m->kv_heads = g.get_int_i32(a + ".attention.head_count_kv", m->heads);
    m->head_dim = g.get_int_i32(a + ".attention.key_length", m->embd / m->heads);
    m->rope_base = g.get_float(a + ".rope.freq_base", 10000.0f);
    m->vocab = g.n_tokens;
    if (!gemma_encoder) {
        m->sliding = g.get_int_i32(a + ".attention.sliding_window", 0);
        m->global_interval = m->sliding > 0 ? 6 : 0;
        m->rope_base_global = m->sliding > 0 ? 1000000.0f : m->rope_base;
    } else {
        m->rope_base_global = m->rope_base;
    }
    if (m->kv_heads <= 0 || m->heads % m->kv_heads || m->head_dim <= 0 || m->head_dim % 2)
        return set_err(ctx, SLX_EINVAL, "bad attention dimensions");
    m->q_dim = m->heads * m->head_dim;
    m->kv_dim = m->kv_heads * m->head_dim;
    Loader ld{ctx, m, g};
    int d = m->embd, F = m->ff, hd = m->head_dim, st;
    const GgufTensor* te = g.tensor("token_embd.weight");
    if (!te) return set_err(ctx, SLX_ENOTFOUND, "Tensor 'token_embd.weight' not found in GGUF file");
    if ((st = ld.weight("token_embd.weight", d, te->elements / d, gemma_encoder ? 0 : 1, m->tok))) return st;
    if ((st = ld.vec_q30("output_norm.weight", d, &m->out_norm))) return st;
    m->L.resize(m->layers);
    for (int i = 0; i < m->layers; i++) {
        std::string p = "blk." + std::to_string(i);
        auto& l = m->L[i];
        if ((st = ld.vec_q30(p + ".attn_norm.weight", d, &l.attn_norm))) return st;
        if ((st = ld.weight(p + ".attn_q.weight", d, m->q_dim, 1, l.q))) return st;
        if ((st = ld.weight(p + ".attn_k.weight", d, m->kv_dim, 1, l.k))) return st;
        if ((st = ld.weight(p + ".attn_v.weight", d, m->kv_dim, 1, l.v))) return st;
        if (gemma_encoder) {
            if ((st = ld.vec_q30(p + ".attn_q_norm.weight", hd, &l.qn))) return st;
            if ((st = ld.vec_q30(p + ".attn_k_norm.weight", hd, &l.kn))) return st;
        } else {
            if ((st = ld.vec_or_ones(p + ".attn_q_norm.weight", hd, &l.qn))) return st;
            if ((st = ld.vec_or_ones(p + ".attn_k_norm.weight", hd, &l.kn))) return st;
        }
        if ((st = ld.weight(p + ".attn_output.weight", m->q_dim, d, 1, l.o))) return st;
        if (gemma_encoder) {
            if ((st = ld.vec_q30(p + ".post_attention_norm.weight", d, &l.post_attn))) return st;
        } else if ((st = ld.vec_or_ones(p + ".post_attention_norm.weight", d, &l.post_attn))) {
            return st;
        }
        if ((st = ld.vec_q30(p + ".ffn_norm.weight", d, &l.ffn_norm))) return st;
        if ((st = ld.weight(p + ".ffn_gate.weight", d, F, 1, l.gate))) return st;
        if ((st = ld.weight(p + ".ffn_up.weight", d, F, 1, l.up))) return st;
        if ((st = ld.weight(p + ".ffn_down.weight", F, d, 1, l.down))) return st;
        if (gemma_encoder) {
            if ((st = ld.vec_q30(p + ".post_ffw_norm.weight", d, &l.post_ffw))) return st;
        } else if ((st = ld.vec_or_ones(p + ".post_ffw_norm.weight", d, &l.post_ffw))) {
            return st;
        }
    }
    m->unk = g.unk; m->eos = g.eos;
    m->rope_rows = 2048;  // RopeMaxSeqLen (IntegerCausalSource.cs:38, IntegerGemmaSource.cs:30)
    if ((st = ld.rope(m->rope_rows, hd, m->rope_base, &m->cos_l, &m->sin_l))) return st;
    return ld.rope(m->rope_rows, hd, m->rope_base_global, &m->cos_g, &m->sin_g);
}

int prepare_gemms(slx_ctx* ctx, slx_model* m) {
    for (auto& l : m->L) {
        WDesc* ws[8] = {&l.qkv, &l.o, &l.gate, &l.up, &l.down, &l.q, &l.k, &l.v};
        GemmPlan* ps[8] = {&l.p_qkv, &l.p_o, &l.p_gate, &l.p_up, &l.p_down, &l.p_q, &l.p_k, &l.p_v};
        for (int i = 0; i < 8; i++) {
            if (!ws[i]->data) continue;
            int st = gemm_prepare(*ws[i], *ps[i], ctx->stream, ctx->err);
            if (st) return st;
            if (ps[i]->limb_bytes) m->allocs.push_back(ps[i]->limbs);
            if (ps[i]->row_shift) m->allocs.push_back(ps[i]->row_shift);
        }
    }
    return SLX_OK;
}

// Attention for one layer: tensor-core scores when the shape allows (exact kernel gated behind).
// q and k are rotated in place first (ApplyRoPE with the cos / sin tables): by the tensor-core path's
// digit split itself, or by k_rope before the exact kernel.
// With planes ([5][mpad][kpad], kpad == nh * hd) the tensor-core path also writes the output rows'
// activation digit planes for the next projection and sets *planes_flag to the word that must stay
// zero for them to be used; otherwise *planes_flag is left null.
int attend(slx_model* m, int64_t* q, int64_t ldq, int64_t* k, int64_t ldk, const int64_t* v, int64_t ldv,
           int64_t* out, int64_t ldo, int B, int T, int nh, int nkv, int hd, int sshift, int64_t sq, int mode, int window,
           const int64_t* cs, const int64_t* sn, cudaStream_t st, int8_t* planes = nullptr, int64_t mpad = 0,
           int64_t kpad = 0, const int** planes_flag = nullptr) {
    if (planes_flag) *planes_flag = nullptr;
    if (tc_enabled() && attention_tc_supported(T, nh, nkv, hd)) {
        size_t need = attention_tc_workspace(B, T, nh, nkv, hd);
        void* ws = m->buf<uint8_t>("attn_ws", need);
        if (ws) {
            const bool pl = planes && planes_flag && kpad == (int64_t)nh * hd && mpad >= (int64_t)B * T;
            int n = attention_tc(q, ldq, k, ldk, v, ldv, out, ldo, B, T, nh, nkv, hd, sshift, sq, mode, window, ws,
                                 m->ctx->d_flag, st, cs, sn, pl ? planes : nullptr, mpad, kpad);
            if (n >= 0) {
                if (pl) *planes_flag = attention_tc_flag(ws);
                return n;
            }
        }
    }
    int n = rope_rows(q, ldq, B, T, nh, hd, cs, sn, st);
    n += rope_rows(k, ldk, B, T, nkv, hd, cs, sn, st);
    return n + attention(q, ldq, k, ldk, v, ldv, out, ldo, B, T, nh, nkv, hd, sshift, sq, mode, window, st);
}

// One projection: c = (a . w^T) >> shift (+ r).
inline void project(slx_model* m, const int64_t* a, int64_t lda, int M, const WDesc& w, const GemmPlan& p, int64_t* c,
                    int64_t ldc, const int64_t* r, int64_t ldr, cudaStream_t st) {
    double macs = (double)M * (double)w.N * (double)w.K;
    // digit products the tensor-core path issues: 5 activation digits x the weight's digits, K padded
    const bool tc_path = p.use_tc && !(!r && gemv_supported(w, M));
    const double tc = tc_path ? (double)M * (double)w.N * (double)p.k_pad * tc::LA * p.wlimbs : 0.0;
    run_k(m->ctx, KC_GEMM, macs, 0, st, [&] { return gemm_run(a, lda, M, w, p, c, ldc, m->scale_bits, r, ldr, m->gws, st); },
          tc);
}
// Projections of the same activations (Q/K/V, gate/up), the activation digits formed once.
inline void project_multi(slx_model* m, const int64_t* a, int64_t lda, int M, int n, const WDesc* const* w,
                          const GemmPlan* const* p, int64_t* const* c, const int64_t* ldc, cudaStream_t st) {
    double macs = 0, tc = 0;
    for (int i = 0; i < n; i++) {
        macs += (double)M * (double)w[i]->N * (double)w[i]->K;
        if (p[i]->use_tc && !gemv_supported(*w[i], M))
            tc += (double)M * (double)w[i]->N * (double)p[i]->k_pad * tc::LA * p[i]->wlimbs;
    }
    run_k(m->ctx, KC_GEMM, macs, 0, st,
          [&] { return gemm_run_multi(a, lda, M, n, w, p, c, ldc, m->scale_bits, m->gws, st); }, tc);
}
// FixedSiLU gate then the down projection (IntegerFFN.Apply, Math/IntegerFFN.cs:70-100): the gate
// kernel writes the down projection's activation digit planes as it writes the gated values, so
// the projection skips its own digit split; shapes it does not cover take the separate kernels.
inline void gate_down(slx_model* m, const int64_t* gate, int64_t* up, int F, int M, const WDesc& w, const GemmPlan& p,
                      int64_t* c, int64_t ldc, const int64_t* r, int64_t ldr, cudaStream_t st) {
    slx_ctx* ctx = m->ctx;
    const int64_t mpad = (M + tc::BM - 1) / tc::BM * tc::BM;
    const bool fused = F % 4 == 0 && p.use_tc && !(!r && gemv_supported(w, M)) && p.k_pad == (F + tc::BK - 1) / tc::BK * tc::BK;
    uint8_t* buf = fused ? m->buf<uint8_t>("down_planes", 256 + (size_t)tc::LA * mpad * p.k_pad) : nullptr;
    if (!buf) {
        run_k(ctx, KC_FFN_GATE, 0, 0, st, [&] { return silu_gate(gate, F, up, F, M, F, st); });
        project(m, up, F, M, w, p, c, ldc, r, ldr, st);
        return;
    }
    int* flag = (int*)buf;
    int8_t* planes = (int8_t*)buf + 256;
    cudaMemsetAsync(flag, 0, sizeof(int), st);
    run_k(ctx, KC_FFN_GATE, 0, 0, st,
          [&] { return silu_gate_digits(gate, F, up, F, M, F, mpad, p.k_pad, planes, flag, st); });
    const double macs = (double)M * (double)w.N * (double)w.K;
    const double tc = (double)M * (double)w.N * (double)p.k_pad * tc::LA * p.wlimbs;
    run_k(ctx, KC_GEMM, macs, 0, st, [&] {
        if (gemm_run_planes(planes, flag, up, F, M, w, p, c, ldc, m->scale_bits, r, ldr, m->gws, st)) return 1;
        return gemm_run(up, F, M, w, p, c, ldc, m->scale_bits, r, ldr, m->gws, st);
    }, tc);
}
// LayerNorm of M rows of d (IntegerLayerNorm.NormalizeRow) that also writes the rows' activation
// digit planes for the projection(s) reading them next. Returns the planes buffer (overflow word at
// byte 0, planes [5][M_pad][K_pad] from byte 256), or nullptr when the plain kernel ran instead.
inline uint8_t* norm_digits(slx_model* m, int64_t* x, int M, int d, const int64_t* w, const int64_t* b, cudaStream_t st) {
    slx_ctx* ctx = m->ctx;
    const int64_t mpad = (M + tc::BM - 1) / tc::BM * tc::BM, kpad = (d + tc::BK - 1) / tc::BK * tc::BK;
    uint8_t* buf = tc_enabled() ? m->buf<uint8_t>("ln_planes", 256 + (size_t)tc::LA * mpad * kpad) : nullptr;
    int n = -1;
    if (buf) {
        cudaMemsetAsync(buf, 0, sizeof(int), st);
        run_k(ctx, KC_NORM, 0, 0, st, [&] {
            n = layernorm_rows_digits(x, d, M, d, w, b, mpad, kpad, (int8_t*)buf + 256, (int*)buf, st);
            return n < 0 ? 0 : n;
        });
    }
    if (n >= 0) return buf;
    run_k(ctx, KC_NORM, 0, 0, st, [&] { return layernorm_rows(x, d, M, d, w, b, st); });
    return nullptr;
}

// A projection of rows whose digit planes a producer wrote (norm_digits, the attention's P.V): the
// planes are used while *flag is zero, the int64 rows by the exact kernel otherwise; the split runs
// itself when there are none or the weight does not take the tensor-core path.
inline void project_from(slx_model* m, const int8_t* planes, const int* flag, const int64_t* a, int64_t lda, int M,
                         const WDesc& w, const GemmPlan& p, int64_t* c, int64_t ldc, const int64_t* r, int64_t ldr,
                         cudaStream_t st) {
    const int64_t kpad = (w.K + tc::BK - 1) / tc::BK * tc::BK;
    if (!planes || p.k_pad != kpad) {
        project(m, a, lda, M, w, p, c, ldc, r, ldr, st);
        return;
    }
    const double macs = (double)M * (double)w.N * (double)w.K;
    const bool tcp = p.use_tc && !(!r && gemv_supported(w, M));
    const double tc = tcp ? (double)M * (double)w.N * (double)p.k_pad * tc::LA * p.wlimbs : 0.0;
    run_k(m->ctx, KC_GEMM, macs, 0, st, [&] {
        if (gemm_run_planes(planes, flag, a, lda, M, w, p, c, ldc, m->scale_bits, r, ldr, m->gws, st))
            return 1;
        return gemm_run(a, lda, M, w, p, c, ldc, m->scale_bits, r, ldr, m->gws, st);
    }, tc);
}
inline void project_from(slx_model* m, const uint8_t* norm_buf, const int64_t* a, int64_t lda, int M, const WDesc& w,
                         const GemmPlan& p, int64_t* c, int64_t ldc, const int64_t* r, int64_t ldr, cudaStream_t st) {
    project_from(m, norm_buf ? (const int8_t*)norm_buf + 256 : nullptr, (const int*)norm_buf, a, lda, M, w, p, c, ldc, r,
                 ldr, st);
}
// Digit planes for the attention output (the O projection's activations), padding rows zeroed; null
// when the tensor-core path is off or the width is not a whole number of 128-byte K blocks.
inline int8_t* attention_planes(slx_model* m, int M, int width, int64_t& mpad, cudaStream_t st) {
    mpad = (M + tc::BM - 1) / tc::BM * tc::BM;
    if (!tc_enabled() || width % tc::BK != 0) return nullptr;
    int8_t* pl = m->buf<int8_t>("att_planes", (size_t)tc::LA * mpad * width);
    if (pl && mpad > M)
        for (int i = 0; i < tc::LA; i++) cudaMemsetAsync(pl + ((int64_t)i * mpad + M) * width, 0, (size_t)(mpad - M) * width, st);
    return pl;
}
#define RUN(cls, macs, bytes, call) run_k(ctx, cls, macs, bytes, st, [&] { return call; })

// Encoder forward to the last block's output, x[B*T][d] (layer limit for tracing).
int encoder_hidden(slx_model* m, const int32_t* ids, int B, int T, int n_layers, int64_t*& x_out, cudaStream_t st) {
    slx_ctx* ctx = m->ctx;
    if (T > m->rope_rows) return set_err(ctx, SLX_ERANGE, "sequence length %d exceeds the RoPE table (%d rows)", T, m->rope_rows);
    const int d = m->embd, F = m->ff, M = B * T, hd = m->head_dim;
    int64_t* x = m->buf<int64_t>("x", (size_t)M * d);
    int64_t* qkv = m->buf<int64_t>("qkv", (size_t)M * 3 * d);
    int64_t* att = m->buf<int64_t>("att", (size_t)M * d);
    int64_t* h = m->buf<int64_t>("h", (size_t)M * d);
    int64_t* gate = m->buf<int64_t>("gate", (size_t)M * F);
    int64_t* up = m->buf<int64_t>("up", (size_t)M * F);
    if (!x || !qkv || !att || !h || !gate || !up) return set_err(ctx, SLX_EOOM, "workspace allocation failed (M=%d)", M);
    RUN(KC_EMBED, 0, 0, embed_encoder(ids, B, T, m->tok, m->tt, m->unk, x, ctx->d_flag, st));
    const uint8_t* xpl = norm_digits(m, x, M, d, m->enw, m->enb, st);  // digit planes of x for the QKV projection
    int64_t apad = 0;
    int8_t* apl = attention_planes(m, M, d, apad, st);  // the P.V writes the O projection's digit planes
    const int sshift = 2 * m->scale_bits - 30;
    const int64_t sq = std::max<int64_t>(1, isqrt64_host(hd));
    int nl = n_layers < 0 ? m->layers : std::min(n_layers, m->layers);
    for (int i = 0; i < nl; i++) {
        auto& l = m->L[i];
        project_from(m, xpl, x, d, M, l.qkv, l.p_qkv, qkv, 3 * d, nullptr, 0, st);
        const int* aflag = nullptr;
        RUN(KC_ATTENTION, 2.0 * B * m->heads * (double)T * T * hd, 0,
            attend(m, qkv, 3 * d, qkv + d, 3 * d, qkv + 2 * d, 3 * d, att, d, B, T, m->heads, m->heads, hd, sshift, sq, 0, 0,
                   m->cos_g, m->sin_g, st, apl, apad, d, &aflag));
        project_from(m, aflag ? apl : nullptr, aflag, att, d, M, l.o, l.p_o, h, d, x, d, st);  // O-projection + residual
        const uint8_t* hpl = norm_digits(m, h, M, d, l.anw, l.anb, st);
        if (hpl) {  // gate and up read the normalised rows' digit planes the norm wrote
            project_from(m, hpl, h, d, M, l.gate, l.p_gate, gate, F, nullptr, 0, st);
            project_from(m, hpl, h, d, M, l.up, l.p_up, up, F, nullptr, 0, st);
        } else {  // one digit split for both
            const WDesc* ws2[2] = {&l.gate, &l.up};
            const GemmPlan* ps2[2] = {&l.p_gate, &l.p_up};
            int64_t* cs2[2] = {gate, up};
            const int64_t ld2[2] = {F, F};
            project_multi(m, h, d, M, 2, ws2, ps2, cs2, ld2, st);
        }
        gate_down(m, gate, up, F, M, l.down, l.p_down, x, d, h, d, st);  // SiLU gate, down-projection + residual
        xpl = norm_digits(m, x, M, d, l.lnw, l.lnb, st);
    }
    x_out = x;
    return SLX_OK;
}

// Causal / Gemma-encoder forward to the last block's output x[B*T][d].
int causal_hidden(slx_model* m, const int32_t* ids, int B, int T, int n_layers, int64_t*& x_out, cudaStream_t st) {
    slx_ctx* ctx = m->ctx;
    if (T > m->rope_rows) return set_err(ctx, SLX_ERANGE, "sequence length %d exceeds the RoPE table (%d rows)", T, m->rope_rows);
    const int d = m->embd, F = m->ff, M = B * T, hd = m->head_dim, qd = m->q_dim, kvd = m->kv_dim;
    int64_t* x = m->buf<int64_t>("x", (size_t)M * d);
    int64_t* xn = m->buf<int64_t>("xn", (size_t)M * d);
    int64_t* p = m->buf<int64_t>("p", (size_t)M * d);
    int64_t* q = m->buf<int64_t>("q", (size_t)M * qd);
    int64_t* k = m->buf<int64_t>("k", (size_t)M * kvd);
    int64_t* v = m->buf<int64_t>("v", (size_t)M * kvd);
    int64_t* att = m->buf<int64_t>("att", (size_t)M * qd);
    int64_t* gate = m->buf<int64_t>("gate", (size_t)M * F);
    int64_t* up = m->buf<int64_t>("up", (size_t)M * F);
    if (!x || !xn || !p || !q || !k || !v || !att || !gate || !up)
        return set_err(ctx, SLX_EOOM, "workspace allocation failed (M=%d)", M);
    const bool causal = m->kind == SLX_MODEL_CAUSAL;
    RUN(KC_EMBED, 0, 0, embed_scaled(ids, B, T, m->tok, m->unk, isqrt64_host(d), x, ctx->d_flag, st));
    int64_t apad = 0;
    int8_t* apl = attention_planes(m, M, qd, apad, st);  // the P.V writes the O projection's digit planes
    const int sshift = 2 * m->scale_bits - 30;
    const int64_t sq = std::max<int64_t>(1, isqrt64_host(hd));
    int nl = n_layers < 0 ? m->layers : std::min(n_layers, m->layers);
    // The norms around each residual add run as one kernel per pair (rms_pair_rows), which also
    // writes the normalised rows' digit planes for the projections that read them (overflow word
    // at byte 0, planes from byte 256); without it, the separate norm, add and copy launches.
    const int64_t npad = (M + tc::BM - 1) / tc::BM * tc::BM;
    uint8_t* nbuf = tc_enabled() ? m->buf<uint8_t>("rms_planes", 256 + (size_t)tc::LA * npad * d) : nullptr;
    int8_t* npl = nbuf ? (int8_t*)nbuf + 256 : nullptr;
    int* nflag = (int*)nbuf;
    auto rms_pair = [&](int64_t* y, const int64_t* r, int64_t* z, const int64_t* w1, const int64_t* w2) -> bool {
        int n = -1;
        if (nbuf && w2) cudaMemsetAsync(nflag, 0, sizeof(int), st);
        RUN(KC_NORM, 0, 0, (n = rms_pair_rows(y, r, z, M, d, w1, w2, npad, d, w2 ? npl : nullptr, nflag, st)) < 0 ? 0 : n);
        return n >= 0;
    };
    bool xn_ready = false;  // xn (and its planes) already hold this layer's pre-attention norm
    for (int i = 0; i < nl; i++) {
        auto& l = m->L[i];
        bool global = !causal || m->global_interval <= 0 || ((i + 1) % m->global_interval) == 0;  // IsGlobalLayer
        bool planes = xn_ready;
        if (!xn_ready) {
            planes = nbuf && rms_pair(x, nullptr, xn, nullptr, l.attn_norm);
            if (!planes) {
                cudaMemcpyAsync(xn, x, sizeof(int64_t) * M * d, cudaMemcpyDeviceToDevice, st);
                RUN(KC_NORM, 0, 0, rmsnorm_rows(xn, d, M, 1, d, l.attn_norm, st));
            }
        }
        xn_ready = false;
        if (planes) {  // Q, K and V read the norm's digit planes
            project_from(m, npl, nflag, xn, d, M, l.q, l.p_q, q, qd, nullptr, 0, st);
            project_from(m, npl, nflag, xn, d, M, l.k, l.p_k, k, kvd, nullptr, 0, st);
            project_from(m, npl, nflag, xn, d, M, l.v, l.p_v, v, kvd, nullptr, 0, st);
        } else {  // Q, K and V read the same normalised rows: one digit split for all three
            const WDesc* ws3[3] = {&l.q, &l.k, &l.v};
            const GemmPlan* ps3[3] = {&l.p_q, &l.p_k, &l.p_v};
            int64_t* cs3[3] = {q, k, v};
            const int64_t ld3[3] = {qd, kvd, kvd};
            project_multi(m, xn, d, M, 3, ws3, ps3, cs3, ld3, st);
        }
        RUN(KC_NORM, 0, 0, rmsnorm_rows(q, qd, M * m->heads, m->heads, hd, l.qn, st));
        RUN(KC_NORM, 0, 0, rmsnorm_rows(k, kvd, M * m->kv_heads, m->kv_heads, hd, l.kn, st));
        const int64_t* cs = global ? m->cos_g : m->cos_l;
        const int64_t* sn = global ? m->sin_g : m->sin_l;
        int mode = !causal ? 0 : ((global || m->sliding <= 0) ? 1 : 2);
        const int* aflag = nullptr;
        RUN(KC_ATTENTION, 2.0 * B * m->heads * (double)T * T * hd, 0,
            attend(m, q, qd, k, kvd, v, kvd, att, qd, B, T, m->heads, m->kv_heads, hd, sshift, sq, mode, m->sliding, cs, sn, st,
                   apl, apad, qd, &aflag));
        project_from(m, aflag ? apl : nullptr, aflag, att, qd, M, l.o, l.p_o, p, d, nullptr, 0, st);
        // p = post-attention norm(p) + x (p is the FFN's residual), xn = ffn_norm(p)
        if (nbuf && rms_pair(p, x, xn, l.post_attn, l.ffn_norm)) {
            project_from(m, npl, nflag, xn, d, M, l.gate, l.p_gate, gate, F, nullptr, 0, st);
            project_from(m, npl, nflag, xn, d, M, l.up, l.p_up, up, F, nullptr, 0, st);
        } else {
            RUN(KC_NORM, 0, 0, rmsnorm_rows(p, d, M, 1, d, l.post_attn, st));
            RUN(KC_ADD, 0, 0, add_rows(p, d, x, d, M, d, st));  // projected += residual; p is the FFN residual
            cudaMemcpyAsync(xn, p, sizeof(int64_t) * M * d, cudaMemcpyDeviceToDevice, st);
            RUN(KC_NORM, 0, 0, rmsnorm_rows(xn, d, M, 1, d, l.ffn_norm, st));
            const WDesc* ws2[2] = {&l.gate, &l.up};
            const GemmPlan* ps2[2] = {&l.p_gate, &l.p_up};
            int64_t* cs2[2] = {gate, up};
            const int64_t ld2[2] = {F, F};
            project_multi(m, xn, d, M, 2, ws2, ps2, cs2, ld2, st);
        }
        gate_down(m, gate, up, F, M, l.down, l.p_down, x, d, nullptr, 0, st);
        // x = post-FFN norm(x) + p, and the next layer's pre-attention norm xn = attn_norm(x)
        const int64_t* next_norm = i + 1 < nl ? m->L[i + 1].attn_norm : nullptr;
        if (nbuf && rms_pair(x, p, xn, l.post_ffw, next_norm)) {
            xn_ready = next_norm != nullptr;
        } else {
            RUN(KC_NORM, 0, 0, rmsnorm_rows(x, d, M, 1, d, l.post_ffw, st));
            RUN(KC_ADD, 0, 0, add_rows(x, d, p, d, M, d, st));
        }
    }
    x_out = x;
    return SLX_OK;
}

// Reads the context's device error word after the work queued on st, clears it (each error is
// reported once) and maps it to a status.
int check_flag(slx_ctx* ctx, cudaStream_t st) {
    int flag = 0;
    CK(cudaMemcpyAsync(&flag, ctx->d_flag, sizeof(int), cudaMemcpyDeviceToHost, st));
    CK(cudaMemsetAsync(ctx->d_flag, 0, sizeof(int), st));
    CK(cudaStreamSynchronize(st));
    if (flag & KERR_RANGE) return set_err(ctx, SLX_ERANGE, "index out of range (token id and UNK row outside the table)");
    if (flag & KERR_TIMEOUT) return set_err(ctx, SLX_ETIMEOUT, "a tensor-core GEMM gave up on a bounded wait");
    return SLX_OK;
}

cudaStream_t pick(slx_ctx* ctx, void* s) { return s ? (cudaStream_t)s : ctx->stream; }

int encode_eager(slx_model* m, const int32_t* d_ids, int B, int T, int64_t* d_pooled, cudaStream_t st);

// The integer encoder's forward replayed from a CUDA graph: the ids are copied into the graph's own
// input buffer and the pooled rows out of its output buffer, so one capture serves every call of
// the same shape. A shape is captured on its second call, after an eager call of that shape that
// allocated nothing further (every buffer at its size); the graph is replayed only while no buffer
// has been reallocated since (the generation count), with the same bounded-wait settings, outside
// profiling (which brackets kernel classes with events) and on a stream other than the legacy one.
// Any failure to capture or instantiate turns graphs off for the model; the eager path computes the
// same result. Sets served when the graph ran the call; returns a status.
int encode_graph(slx_model* m, const int32_t* d_ids, int B, int T, int64_t* d_pooled, cudaStream_t st, bool& served) {
    slx_ctx* ctx = m->ctx;
    auto& g = m->eg;
    served = false;
    if (g.disabled || ctx->prof || !st || m->kind != SLX_MODEL_ENCODER || !tc_enabled() || (int64_t)B * T < 64)
        return SLX_OK;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
        cudaGetLastError();
        return SLX_OK;
    }
    int32_t* gids = m->buf<int32_t>("graph_ids", (size_t)B * T);
    int64_t* gout = m->buf<int64_t>("graph_pooled", (size_t)B * m->embd);
    if (!gids || !gout) return SLX_OK;
    const uint64_t gen = m->gen();
    const bool same_wait = g.wait_limit == ctx->wait.limit_cycles && g.stall == ctx->wait.stall_mma;
    if (!(g.exec && g.B == B && g.T == T && g.gen == gen && same_wait)) {
        if (!(g.seen_B == B && g.seen_T == T && g.seen_gen == gen)) return SLX_OK;  // warm this shape eagerly first
        if (g.exec) cudaGraphExecDestroy(g.exec);
        g.exec = nullptr;
        g.B = g.T = -1;
        const int64_t l0 = ctx->launches;
        cudaGraph_t graph = nullptr;
        if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
            cudaGetLastError();
            g.disabled = true;
            return SLX_OK;
        }
        const int rc = encode_eager(m, gids, B, T, gout, st);
        const cudaError_t e = cudaStreamEndCapture(st, &graph);
        const int64_t n = ctx->launches - l0;
        ctx->launches = l0;  // nothing ran during the capture
        cudaGraphExec_t exec = nullptr;
        if (rc != SLX_OK || e != cudaSuccess || !graph || m->gen() != gen ||
            cudaGraphInstantiate(&exec, graph, 0) != cudaSuccess) {
            if (graph) cudaGraphDestroy(graph);
            cudaGetLastError();
            ctx->err.clear();
            g.disabled = true;
            return SLX_OK;
        }
        cudaGraphDestroy(graph);
        g.exec = exec;
        g.B = B;
        g.T = T;
        g.gen = gen;
        g.wait_limit = ctx->wait.limit_cycles;
        g.stall = ctx->wait.stall_mma;
        g.launches = n;
    }
    CK(cudaMemcpyAsync(gids, d_ids, sizeof(int32_t) * B * T, cudaMemcpyDeviceToDevice, st));
    CK(cudaGraphLaunch(g.exec, st));
    CK(cudaMemcpyAsync(d_pooled, gout, sizeof(int64_t) * B * m->embd, cudaMemcpyDeviceToDevice, st));
    ctx->launches += g.launches;
    served = true;
    return SLX_OK;
}

int encode_device(slx_model* m, const int32_t* d_ids, int B, int T, int64_t* d_pooled, cudaStream_t st) {
    slx_ctx* ctx = m->ctx;
    if (B < 0 || T < 0) return set_err(ctx, SLX_EINVAL, "bad batch shape B=%d T=%d", B, T);
    if (B == 0) return SLX_OK;
    if (T == 0) {  // MeanPool of an empty sequence returns zeros (IntegerTransformerSource.Forward.cs:73)
        CK(cudaMemsetAsync(d_pooled, 0, sizeof(int64_t) * B * m->embd, st));
        return SLX_OK;
    }
    bool served = false;
    const int gr = encode_graph(m, d_ids, B, T, d_pooled, st, served);
    if (gr != SLX_OK || served) return gr;
    const int rc = encode_eager(m, d_ids, B, T, d_pooled, st);
    if (rc == SLX_OK) {  // the shape is warm once this call has allocated what it needs
        m->eg.seen_B = B;
        m->eg.seen_T = T;
        m->eg.seen_gen = m->gen();
    }
    return rc;
}

int encode_eager(slx_model* m, const int32_t* d_ids, int B, int T, int64_t* d_pooled, cudaStream_t st) {
    slx_ctx* ctx = m->ctx;
    int64_t* x = nullptr;
    int rc;
    if (m->kind == SLX_MODEL_ENCODER) {
        rc = encoder_hidden(m, d_ids, B, T, -1, x, st);
        if (rc) return rc;
    } else {
        rc = causal_hidden(m, d_ids, B, T, -1, x, st);
        if (rc) return rc;
        RUN(KC_NORM, 0, 0, rmsnorm_rows(x, m->embd, B * T, 1, m->embd, m->out_norm, st));  // final RmsNorm (IntegerGemmaSource.cs:77)
    }
    RUN(KC_POOL, 0, 0, mean_pool(x, m->embd, B, T, m->embd, d_pooled, st));
    CK(cudaGetLastError());
    return SLX_OK;
}

// Last position after the output norm for each of B sequences: last[B][d].
int causal_last(slx_model* m, const int32_t* d_ids, int B, int T, int64_t* d_last, cudaStream_t st) {
    slx_ctx* ctx = m->ctx;
    int64_t* x = nullptr;
    int rc = causal_hidden(m, d_ids, B, T, -1, x, st);
    if (rc) return rc;
    RUN(KC_POOL, 0, 0, gather_last_rows(x, m->embd, B, T, m->embd, d_last, st));
    RUN(KC_NORM, 0, 0, rmsnorm_rows(d_last, m->embd, B, 1, m->embd, m->out_norm, st));
    CK(cudaGetLastError());
    return SLX_OK;
}

// ForwardFloat + L2Normalize on the host (IntegerTransformerSource.cs:52-62, .Forward.cs:89-99):
// sequential fp32 without contraction (the host compiler runs with -ffp-contract=off).
void to_float_l2(const int64_t* v, int d, int sb, float* out) {
    double scale = std::pow(2.0, -sb);
    for (int j = 0; j < d; j++) out[j] = (float)((double)v[j] * scale);
    float norm = 0.0f;
    for (int j = 0; j < d; j++) norm += out[j] * out[j];
    norm = std::sqrt(norm);
    if (norm < 1e-10f) return;
    float inv = 1.0f / norm;
    for (int j = 0; j < d; j++) out[j] *= inv;
}

}  // namespace

// ==============================================================================================
// extern "C" ABI
// ==============================================================================================
extern "C" {

const char* slx_version(void) { return "slx 0.1 (sm_100a)"; }

slx_status slx_init(int device, slx_ctx** out) {
    if (!out) return SLX_EINVAL;
    *out = nullptr;
    std::unique_ptr<slx_ctx> c(new slx_ctx());
    slx_ctx* ctx = c.get();
    c->device = device;
    CK(cudaSetDevice(device));
    CK(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    CK(cudaMalloc(&c->d_flag, sizeof(int)));
    CK(cudaMemset(c->d_flag, 0, sizeof(int)));
    c->kws.wait = &c->wait;
    *out = c.release();
    return SLX_OK;
}

// Drops one reference; the last one frees the context. Models, weights and lattices hold one each,
// so the context (its device, stream and error word) outlives every object created on it, whatever
// order the host frees them in (a garbage-collected host may finalize the context first).
static void ctx_release(slx_ctx* ctx) {
    if (ctx->refs.fetch_sub(1) != 1) return;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->d_flag);
    for (auto& r : ctx->records) { cudaEventDestroy(r.a); cudaEventDestroy(r.b); }
    for (cudaEvent_t e : ctx->event_pool) cudaEventDestroy(e);
    gemm_workspace_free(ctx->kws);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
}

slx_status slx_destroy(slx_ctx* ctx) {
    if (!ctx) return SLX_EINVAL;
    ctx_release(ctx);
    return SLX_OK;
}

const char* slx_last_error(slx_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

slx_status slx_ctx_status(slx_ctx* ctx, void* stream) {
    if (!ctx) return SLX_EINVAL;
    CK(cudaSetDevice(ctx->device));
    return check_flag(ctx, pick(ctx, stream));
}

slx_status slx_ctx_set_option(slx_ctx* ctx, int option, int64_t value) {
    if (!ctx) return SLX_EINVAL;
    switch (option) {
        case SLX_OPT_WAIT_LIMIT_CYCLES:
            if (value < 0) return set_err(ctx, SLX_EINVAL, "wait limit %lld < 0", (long long)value);
            ctx->wait.limit_cycles = value;
            return SLX_OK;
        case SLX_OPT_TEST_STALL_MMA:
            ctx->wait.stall_mma = value ? 1 : 0;
            return SLX_OK;
        default:
            return set_err(ctx, SLX_EINVAL, "unknown option %d", option);
    }
}

slx_status slx_model_load_gguf(slx_ctx* ctx, const char* path, int kind, int scale_bits, slx_model** out) {
    if (!ctx || !path || !out) return set_err(ctx, SLX_EINVAL, "null argument");
    *out = nullptr;
    if (scale_bits < 1 || scale_bits > 62) return set_err(ctx, SLX_EINVAL, "scale_bits %d out of range", scale_bits);
    CK(cudaSetDevice(ctx->device));
    GgufFile g;
    std::string err;
    int st = g.open(path, err);
    if (st) return set_err(ctx, st, "%s", err.c_str());
    std::unique_ptr<slx_model> m(new slx_model());
    m->ctx = ctx;
    m->kind = kind;
    m->scale_bits = scale_bits;
    if (kind == SLX_MODEL_ENCODER)
        st = load_encoder(ctx, m.get(), g);
    else if (kind == SLX_MODEL_CAUSAL || kind == SLX_MODEL_GEMMA_ENCODER)
        st = load_causal(ctx, m.get(), g, kind == SLX_MODEL_GEMMA_ENCODER);
    else if (kind == SLX_MODEL_FLOAT_ENCODER)
        st = load_float_encoder(ctx, m.get(), g);
    else
        return set_err(ctx, SLX_EINVAL, "unknown model kind %d", kind);
    if (st) return st;
    m->gws.err = ctx->d_flag;
    m->gws.wait = &ctx->wait;
    if ((st = prepare_gemms(ctx, m.get()))) return st;
    CK(cudaStreamSynchronize(ctx->stream));
    CK(cudaGetLastError());
    ctx->refs.fetch_add(1);
    *out = m.release();
    return SLX_OK;
}

slx_status slx_model_free(slx_model* m) {
    if (!m) return SLX_EINVAL;
    slx_ctx* ctx = m->ctx;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    delete m;
    ctx_release(ctx);
    return SLX_OK;
}

slx_status slx_model_info(slx_model* m, int32_t* info, int n) {
    if (!m || !info) return SLX_EINVAL;
    int32_t v[12] = {m->kind, m->embd, m->heads, m->kv_heads, m->head_dim, m->ff, m->layers, m->vocab, m->eos, m->unk,
                     m->q_dim, m->kv_dim};
    for (int i = 0; i < n && i < 12; i++) info[i] = v[i];
    return SLX_OK;
}

slx_status slx_encode_device(slx_model* m, const int32_t* d_ids, int B, int T, int64_t* d_pooled, void* stream) {
    if (!m || (B > 0 && T > 0 && (!d_ids || !d_pooled))) return m ? set_err(m->ctx, SLX_EINVAL, "null argument") : SLX_EINVAL;
    if (m->kind == SLX_MODEL_CAUSAL) return set_err(m->ctx, SLX_EINVAL, "slx_encode on a causal model");
    if (m->kind == SLX_MODEL_FLOAT_ENCODER) return set_err(m->ctx, SLX_EINVAL, "the float encoder has no Q30 output");
    return encode_device(m, d_ids, B, T, d_pooled, pick(m->ctx, stream));
}

// TransformerEmbeddingSource.Forward / EmbedBatchAsync (Gguf/TransformerEmbeddingSource.cs:106-141) for B
// sequences of T ids: L2-normalised float embeddings.
static slx_status encode_float(slx_model* m, const int32_t* ids, int B, int T, float* out) {
    slx_ctx* ctx = m->ctx;
    if (T > m->rope_rows)
        return set_err(ctx, SLX_ERANGE, "sequence length %d exceeds the RoPE table (%d rows)", T, m->rope_rows);
    if (B == 0) return SLX_OK;
    CK(cudaSetDevice(ctx->device));
    cudaStream_t st = ctx->stream;
    int32_t* d_ids = m->buf<int32_t>("ids", (size_t)std::max(1, B * T));
    float* d_out = m->buf<float>("fout", (size_t)B * m->embd);
    if (!d_ids || !d_out) return set_err(ctx, SLX_EOOM, "workspace allocation failed");
    if (T == 0) {  // MeanPool of no rows is the zero vector, which L2Normalize leaves unchanged
        std::fill(out, out + (size_t)B * m->embd, 0.0f);
        return SLX_OK;
    }
    CK(cudaMemcpyAsync(d_ids, ids, sizeof(int32_t) * B * T, cudaMemcpyHostToDevice, st));
    int rc = 0;
    run_k(ctx, KC_GEMM, (double)B * T * (3.0 * m->embd * m->embd + m->embd * m->embd + 3.0 * m->embd * m->ff) * m->fm.layers.size(),
          0, st, [&] {
              const int n = fenc::forward(m->fm, d_ids, B, T, d_out, m->fws, st, nullptr);
              if (n < 0) rc = SLX_EOOM;
              return n < 0 ? 0 : n;
          });
    if (rc) return set_err(ctx, rc, "workspace allocation failed");
    CK(cudaMemcpyAsync(out, d_out, sizeof(float) * B * m->embd, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    return SLX_OK;
}

slx_status slx_encode(slx_model* m, const int32_t* ids, int B, int T, int64_t* pooled, float* l2) {
    if (!m) return SLX_EINVAL;
    slx_ctx* ctx = m->ctx;
    if (m->kind == SLX_MODEL_FLOAT_ENCODER) {
        if (B < 0 || T < 0 || (B > 0 && T > 0 && !ids) || (B > 0 && !l2) || pooled)
            return set_err(ctx, SLX_EINVAL, "bad arguments (the float encoder fills l2 only)");
        return encode_float(m, ids, B, T, l2);
    }
    if (B < 0 || T < 0 || (B > 0 && T > 0 && !ids) || (B > 0 && !pooled)) return set_err(ctx, SLX_EINVAL, "bad arguments");
    if (m->kind == SLX_MODEL_CAUSAL) return set_err(ctx, SLX_EINVAL, "slx_encode on a causal model");
    if (B == 0) return SLX_OK;
    CK(cudaSetDevice(ctx->device));
    cudaStream_t st = ctx->stream;
    int32_t* d_ids = m->buf<int32_t>("ids", (size_t)std::max(1, B * T));
    int64_t* d_pooled = m->buf<int64_t>("pooled", (size_t)B * m->embd);
    if (!d_ids || !d_pooled) return set_err(ctx, SLX_EOOM, "workspace allocation failed");
    CK(cudaMemsetAsync(ctx->d_flag, 0, sizeof(int), st));
    if (B * T > 0) CK(cudaMemcpyAsync(d_ids, ids, sizeof(int32_t) * B * T, cudaMemcpyHostToDevice, st));
    int rc = encode_device(m, d_ids, B, T, d_pooled, st);
    if (rc) return rc;
    CK(cudaMemcpyAsync(pooled, d_pooled, sizeof(int64_t) * B * m->embd, cudaMemcpyDeviceToHost, st));
    if ((rc = check_flag(ctx, st))) return rc;
    if (l2)
        for (int b = 0; b < B; b++) to_float_l2(pooled + (int64_t)b * m->embd, m->embd, m->scale_bits, l2 + (int64_t)b * m->embd);
    return SLX_OK;
}

slx_status slx_trace_hidden(slx_model* m, const int32_t* ids, int T, int n_layers, int final_norm, int64_t* x_q30) {
    if (!m || !ids || !x_q30 || T <= 0) return m ? set_err(m->ctx, SLX_EINVAL, "bad arguments") : SLX_EINVAL;
    slx_ctx* ctx = m->ctx;
    if (m->kind == SLX_MODEL_FLOAT_ENCODER) return set_err(ctx, SLX_EINVAL, "the float encoder has no Q30 trace");
    CK(cudaSetDevice(ctx->device));
    cudaStream_t st = ctx->stream;
    int32_t* d_ids = m->buf<int32_t>("ids", (size_t)T);
    if (!d_ids) return set_err(ctx, SLX_EOOM, "workspace allocation failed");
    CK(cudaMemsetAsync(ctx->d_flag, 0, sizeof(int), st));
    CK(cudaMemcpyAsync(d_ids, ids, sizeof(int32_t) * T, cudaMemcpyHostToDevice, st));
    int64_t* x = nullptr;
    int rc = m->kind == SLX_MODEL_ENCODER ? encoder_hidden(m, d_ids, 1, T, n_layers, x, st)
                                          : causal_hidden(m, d_ids, 1, T, n_layers, x, st);
    if (rc) return rc;
    if (final_norm && m->kind != SLX_MODEL_ENCODER) rmsnorm_rows(x, m->embd, T, 1, m->embd, m->out_norm, st);
    CK(cudaMemcpyAsync(x_q30, x, sizeof(int64_t) * T * m->embd, cudaMemcpyDeviceToHost, st));
    return check_flag(ctx, st);
}

slx_status slx_causal_forward_last(slx_model* m, const int32_t* ids, int T, int64_t* last) {
    if (!m || !ids || !last || T <= 0) return m ? set_err(m->ctx, SLX_EINVAL, "bad arguments") : SLX_EINVAL;
    slx_ctx* ctx = m->ctx;
    if (m->kind != SLX_MODEL_CAUSAL) return set_err(ctx, SLX_EINVAL, "not a causal model");
    CK(cudaSetDevice(ctx->device));
    cudaStream_t st = ctx->stream;
    int32_t* d_ids = m->buf<int32_t>("ids", (size_t)T);
    int64_t* d_last = m->buf<int64_t>("last", (size_t)m->embd);
    if (!d_ids || !d_last) return set_err(ctx, SLX_EOOM, "workspace allocation failed");
    CK(cudaMemsetAsync(ctx->d_flag, 0, sizeof(int), st));
    CK(cudaMemcpyAsync(d_ids, ids, sizeof(int32_t) * T, cudaMemcpyHostToDevice, st));
    int rc = causal_last(m, d_ids, 1, T, d_last, st);
    if (rc) return rc;
    CK(cudaMemcpyAsync(last, d_last, sizeof(int64_t) * m->embd, cudaMemcpyDeviceToHost, st));
    return check_flag(ctx, st);
}

// Builds the VocabLattice of a causal model once (IntegerCausalSource.GetVocabLattice, :69-74).
static int vocab_lattice_ready(slx_model* m, cudaStream_t st) {
    if (m->vlat_ready) return SLX_OK;
    std::string err;
    int rc = vocab::build(m->tok, m->vocab, m->embd, m->vlat, st, err);
    if (rc) return set_err(m->ctx, rc, "%s", err.c_str());
    m->ctx->launches += m->vlat.V > 0 ? 2 : 0;  // table and row norms
    m->vlat_ready = true;
    return SLX_OK;
}

// PredictNextToken (IntegerCausalSource.cs:149-157) for B sequences: the brute-force argmax head
// (lattice_k < 0) or the VocabLattice head with k candidates.
static slx_status causal_next(slx_model* m, const int32_t* ids, int B, int T, int lattice_k, int32_t* next) {
    if (!m || !ids || !next || B <= 0 || T <= 0) return m ? set_err(m->ctx, SLX_EINVAL, "bad arguments") : SLX_EINVAL;
    slx_ctx* ctx = m->ctx;
    if (m->kind != SLX_MODEL_CAUSAL) return set_err(ctx, SLX_EINVAL, "not a causal model");
    if (lattice_k > vocab::KMAX) return set_err(ctx, SLX_EINVAL, "lattice k %d exceeds %d", lattice_k, vocab::KMAX);
    CK(cudaSetDevice(ctx->device));
    cudaStream_t st = ctx->stream;
    int32_t* d_ids = m->buf<int32_t>("ids", (size_t)B * T);
    int64_t* d_last = m->buf<int64_t>("last", (size_t)B * m->embd);
    unsigned long long* keys = m->buf<unsigned long long>("keys", (size_t)B);
    int32_t* d_next = m->buf<int32_t>("next", (size_t)B);
    if (!d_ids || !d_last || !keys || !d_next) return set_err(ctx, SLX_EOOM, "workspace allocation failed");
    const bool lattice = lattice_k >= 0;
    if (lattice) {
        if (int rc = vocab_lattice_ready(m, st)) return rc;
        std::string err;
        if (int rc = vocab::reserve(m->vlat, B, lattice_k, err)) return set_err(ctx, rc, "%s", err.c_str());
    }
    CK(cudaMemsetAsync(ctx->d_flag, 0, sizeof(int), st));
    CK(cudaMemcpyAsync(d_ids, ids, sizeof(int32_t) * B * T, cudaMemcpyHostToDevice, st));
    int rc = causal_last(m, d_ids, B, T, d_last, st);
    if (rc) return rc;
    if (lattice)
        RUN(KC_VOCAB, (double)B * m->vlat.V * m->embd, 0,
            vocab::next_tokens(m->vlat, d_last, B, m->scale_bits, lattice_k, m->eos, d_next, st));
    else
        RUN(KC_ARGMAX, 0, 0, argmax_vocab(d_last, B, m->embd, m->tok, m->vocab, m->scale_bits, keys, d_next, st));
    CK(cudaMemcpyAsync(next, d_next, sizeof(int32_t) * B, cudaMemcpyDeviceToHost, st));
    return check_flag(ctx, st);
}

// Generate (IntegerCausalSource.cs:86-108) on token ids for B sequences: full re-forward per step,
// stop at EOS (not appended).
static slx_status causal_generate(slx_model* m, const int32_t* ids, int B, int T, int max_new, int lattice_k,
                                  int32_t* out, int32_t* n_out) {
    if (!m || !ids || !out || !n_out || B <= 0 || T <= 0 || max_new < 0)
        return m ? set_err(m->ctx, SLX_EINVAL, "bad arguments") : SLX_EINVAL;
    slx_ctx* ctx = m->ctx;
    if (m->kind != SLX_MODEL_CAUSAL) return set_err(ctx, SLX_EINVAL, "not a causal model");
    std::vector<int32_t> seq((size_t)B * T);
    std::memcpy(seq.data(), ids, sizeof(int32_t) * B * T);
    std::vector<int> done((size_t)B, 0);
    for (int b = 0; b < B; b++) n_out[b] = 0;
    std::vector<int32_t> next((size_t)B);
    int cur = T;
    for (int step = 0; step < max_new; step++) {
        int alive = 0;
        for (int b = 0; b < B; b++) alive += !done[b];
        if (!alive) break;
        int rc = causal_next(m, seq.data(), B, cur, lattice_k, next.data());
        if (rc) return rc;
        std::vector<int32_t> grown((size_t)B * (cur + 1));
        for (int b = 0; b < B; b++) {
            std::memcpy(&grown[(size_t)b * (cur + 1)], &seq[(size_t)b * cur], sizeof(int32_t) * cur);
            int32_t nx = next[b];
            if (!done[b] && nx == m->eos) done[b] = 1;  // Generate stops before appending EOS
            if (!done[b]) out[(size_t)b * max_new + n_out[b]++] = nx;
            grown[(size_t)b * (cur + 1) + cur] = done[b] ? m->eos : nx;
        }
        seq.swap(grown);
        cur++;
    }
    return SLX_OK;
}

slx_status slx_causal_next_token(slx_model* m, const int32_t* ids, int B, int T, int32_t* next) {
    return causal_next(m, ids, B, T, -1, next);
}

slx_status slx_causal_next_token_lattice(slx_model* m, const int32_t* ids, int B, int T, int k, int32_t* next) {
    return causal_next(m, ids, B, T, k < 0 ? 0 : k, next);
}

slx_status slx_causal_generate(slx_model* m, const int32_t* ids, int B, int T, int max_new, int32_t* out,
                               int32_t* n_out) {
    return causal_generate(m, ids, B, T, max_new, -1, out, n_out);
}

slx_status slx_causal_generate_lattice(slx_model* m, const int32_t* ids, int B, int T, int max_new, int k,
                                       int32_t* out, int32_t* n_out) {
    return causal_generate(m, ids, B, T, max_new, k < 0 ? 0 : k, out, n_out);
}

slx_status slx_vocab_lattice_query(slx_model* m, const float* hidden, int B, int k, int32_t* ids, uint64_t* dist) {
    if (!m || B < 0 || (B > 0 && k > 0 && (!hidden || !ids)))
        return m ? set_err(m->ctx, SLX_EINVAL, "bad arguments") : SLX_EINVAL;
    slx_ctx* ctx = m->ctx;
    if (m->kind != SLX_MODEL_CAUSAL) return set_err(ctx, SLX_EINVAL, "not a causal model");
    if (k > vocab::KMAX) return set_err(ctx, SLX_EINVAL, "lattice k %d exceeds %d", k, vocab::KMAX);
    if (B == 0 || k <= 0) return SLX_OK;  // QueryKNearestL2 with k <= 0 is empty
    CK(cudaSetDevice(ctx->device));
    cudaStream_t st = ctx->stream;
    if (int rc = vocab_lattice_ready(m, st)) return rc;
    std::string err;
    if (int rc = vocab::reserve(m->vlat, B, k, err)) return set_err(ctx, rc, "%s", err.c_str());
    int32_t* d_ids = m->buf<int32_t>("lattice_ids", (size_t)B * k);
    uint64_t* d_dist = dist ? m->buf<uint64_t>("lattice_dist", (size_t)B * k) : nullptr;
    if (!d_ids || (dist && !d_dist)) return set_err(ctx, SLX_EOOM, "workspace allocation failed");
    CK(cudaMemcpyAsync(m->vlat.hf, hidden, sizeof(float) * (size_t)B * m->embd, cudaMemcpyHostToDevice, st));
    RUN(KC_VOCAB, (double)B * m->vlat.V * m->embd, 0, vocab::query_topk(m->vlat, B, k, d_ids, d_dist, st));
    CK(cudaMemcpyAsync(ids, d_ids, sizeof(int32_t) * (size_t)B * k, cudaMemcpyDeviceToHost, st));
    if (dist) CK(cudaMemcpyAsync(dist, d_dist, sizeof(uint64_t) * (size_t)B * k, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    return SLX_OK;
}

slx_status slx_dequantize(slx_ctx* ctx, int dtype, const uint8_t* raw, int64_t nbytes, float* out, int64_t n) {
    if (!ctx || (n > 0 && (!raw || !out)) || n < 0 || nbytes < 0) return set_err(ctx, SLX_EINVAL, "bad arguments");
    int64_t need = gguf_decode_bytes((uint32_t)dtype, n);
    if (need < 0) return set_err(ctx, SLX_EUNSUPPORTED, "Dequantization of dtype %d is not yet implemented", dtype);
    if (nbytes < need) return set_err(ctx, SLX_EEOF, "Unexpected end of GGUF stream: expected %lld bytes, got %lld", (long long)need, (long long)nbytes);
    if (n == 0) return SLX_OK;
    CK(cudaSetDevice(ctx->device));
    cudaStream_t st = ctx->stream;
    uint8_t* d_raw = nullptr;
    float* d_out = nullptr;
    CK(cudaMalloc(&d_raw, std::max<int64_t>(need, 1)));
    if (cudaMalloc(&d_out, sizeof(float) * n) != cudaSuccess) {
        cudaFree(d_raw);
        return set_err(ctx, SLX_EOOM, "device allocation failed");
    }
    cudaMemsetAsync(ctx->d_flag, 0, sizeof(int), st);
    cudaMemcpyAsync(d_raw, raw, need, cudaMemcpyHostToDevice, st);
    dequant_f32(dtype, d_raw, n, d_out, ctx->d_flag, st);
    cudaMemcpyAsync(out, d_out, sizeof(float) * n, cudaMemcpyDeviceToHost, st);
    int rc = check_flag(ctx, st);
    cudaFree(d_raw);
    cudaFree(d_out);
    return rc;
}

slx_status slx_gguf_read_f32(slx_ctx* ctx, const char* path, const char* tensor, float* out, int64_t n) {
    if (!ctx || !path || !tensor) return set_err(ctx, SLX_EINVAL, "null argument");
    GgufFile g;
    std::string err;
    int st = g.open(path, err);
    if (st) return set_err(ctx, st, "%s", err.c_str());
    const GgufTensor* t = g.tensor(tensor);
    if (!t) return set_err(ctx, SLX_ENOTFOUND, "Tensor '%s' not found in GGUF file", tensor);
    if (n != t->elements) return set_err(ctx, SLX_EINVAL, "output holds %lld floats, tensor has %lld", (long long)n, (long long)t->elements);
    std::vector<uint8_t> raw;
    if ((st = g.read_raw(*t, raw, err))) return set_err(ctx, st, "%s", err.c_str());
    return slx_dequantize(ctx, (int)t->dtype, raw.data(), (int64_t)raw.size(), out, n);
}

slx_status slx_matmul_q30_device(slx_ctx* ctx, const int64_t* d_a, int M, int K, int dtype, const uint8_t* d_w,
                                 int64_t w_bytes, int N, int half_composite, int scale_bits, int shift, int64_t* d_c,
                                 void* stream) {
    if (!ctx || M < 0 || K <= 0 || N <= 0 || !d_w || (M > 0 && (!d_a || !d_c))) return set_err(ctx, SLX_EINVAL, "bad arguments");
    if (dtype != GG_F32 && dtype != GG_F16 && dtype != GG_BF16 && dtype != GG_Q8_0 && dtype != GG_Q4_0)
        return set_err(ctx, SLX_EUNSUPPORTED, "matmul weight dtype %d (expand other formats with slx_dequantize)", dtype);
    int64_t elems = (int64_t)N * K;
    if (w_bytes < gguf_byte_count((uint32_t)dtype, elems)) return set_err(ctx, SLX_EEOF, "weight buffer too small");
    WDesc w;
    w.dtype = dtype; w.data = d_w; w.nblocks = elems / 32; w.elements = elems; w.N = N; w.K = K;
    w.mode = half_composite ? 1 : 0;
    w.scale = std::ldexp(1.0, scale_bits);
    cudaStream_t st = pick(ctx, stream);
    if (gemv_supported(w, M)) {  // decode-shaped: packed-block GEMV, queued without a host sync
        if (!gemv_reserve(ctx->kws, M, N, K, st)) return set_err(ctx, SLX_EOOM, "GEMV workspace");
        ctx->kws.err = ctx->d_flag;
        RUN(KC_GEMV, (double)M * N * K, (double)gguf_byte_count((uint32_t)dtype, elems) + (double)M * (K + N) * 8,
            gemv_exact(d_a, K, M, w, d_c, N, shift, ctx->kws, st));
        CK(cudaGetLastError());
        return SLX_OK;
    }
    // One-off plan: the weight's digit planes are built for this call and released with it.
    GemmPlan plan;
    std::string err;
    int rc = gemm_prepare(w, plan, st, err);
    if (rc) return set_err(ctx, rc, "%s", err.c_str());
    GemmWorkspace ws;
    ws.err = ctx->d_flag;
    ws.wait = &ctx->wait;
    RUN(KC_GEMM, (double)M * N * K, 0, gemm_run(d_a, K, M, w, plan, d_c, N, shift, nullptr, 0, ws, st));
    cudaError_t e = cudaStreamSynchronize(st);
    if (plan.limbs) cudaFree(plan.limbs);
    if (plan.row_shift) cudaFree(plan.row_shift);
    gemm_workspace_free(ws);
    if (e != cudaSuccess) return set_err(ctx, SLX_ECUDA, "%s", cudaGetErrorString(e));
    CK(cudaGetLastError());
    return SLX_OK;
}

// A weight prepared once for repeated products: the load-time half of the reference's weight
// handling (IntegerTransformerSource.Loading.cs:105-119 re-quantizes every weight to Q30 long[] at
// load), here the tensor-core digit planes of the composites, built beside the caller's blocks.
struct slx_weight {
    slx_ctx* ctx = nullptr;
    WDesc w;
    GemmPlan plan;
    GemmWorkspace ws;
    ~slx_weight() {
        if (plan.limbs) cudaFree(plan.limbs);
        if (plan.row_shift) cudaFree(plan.row_shift);
        gemm_workspace_free(ws);
    }
};

slx_status slx_weight_prepare(slx_ctx* ctx, const uint8_t* d_w, int64_t w_bytes, int dtype, int N, int K,
                              int half_composite, int scale_bits, slx_weight** out) {
    if (!ctx || !d_w || !out || N <= 0 || K <= 0 || scale_bits < 1 || scale_bits > 62)
        return set_err(ctx, SLX_EINVAL, "bad arguments");
    *out = nullptr;
    if (dtype != GG_F32 && dtype != GG_F16 && dtype != GG_BF16 && dtype != GG_Q8_0 && dtype != GG_Q4_0)
        return set_err(ctx, SLX_EUNSUPPORTED, "matmul weight dtype %d (expand other formats with slx_dequantize)", dtype);
    const int64_t elems = (int64_t)N * K;
    if (w_bytes < gguf_byte_count((uint32_t)dtype, elems)) return set_err(ctx, SLX_EEOF, "weight buffer too small");
    CK(cudaSetDevice(ctx->device));
    std::unique_ptr<slx_weight> h(new slx_weight());
    h->ctx = ctx;
    WDesc& w = h->w;
    w.dtype = dtype; w.data = d_w; w.nblocks = elems / 32; w.elements = elems; w.N = N; w.K = K;
    w.mode = half_composite ? 1 : 0;
    w.scale = std::ldexp(1.0, scale_bits);
    h->ws.err = ctx->d_flag;
    h->ws.wait = &ctx->wait;
    std::string err;
    int rc = gemm_prepare(w, h->plan, ctx->stream, err);
    if (rc) return set_err(ctx, rc, "%s", err.c_str());
    CK(cudaStreamSynchronize(ctx->stream));
    ctx->refs.fetch_add(1);
    *out = h.release();
    return SLX_OK;
}

slx_status slx_weight_free(slx_weight* w) {
    if (!w) return SLX_EINVAL;
    slx_ctx* ctx = w->ctx;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    delete w;
    ctx_release(ctx);
    return SLX_OK;
}

slx_status slx_weight_info(slx_weight* w, int32_t* info, int n) {
    if (!w || !info) return SLX_EINVAL;
    int32_t v[4] = {(int32_t)w->w.N, (int32_t)w->w.K, w->plan.use_tc, w->plan.wlimbs};
    for (int i = 0; i < n && i < 4; i++) info[i] = v[i];
    return SLX_OK;
}

slx_status slx_matmul_q30_prepared(slx_weight* h, const int64_t* d_a, int M, int shift, int64_t* d_c, void* stream) {
    if (!h) return SLX_EINVAL;
    slx_ctx* ctx = h->ctx;
    if (M < 0 || (M > 0 && (!d_a || !d_c))) return set_err(ctx, SLX_EINVAL, "bad arguments");
    if (M == 0) return SLX_OK;
    cudaStream_t st = pick(ctx, stream);
    const WDesc& w = h->w;
    const double macs = (double)M * (double)w.N * (double)w.K;
    if (gemv_supported(w, M)) {
        if (!gemv_reserve(h->ws, M, (int)w.N, (int)w.K, st)) return set_err(ctx, SLX_EOOM, "GEMV workspace");
        RUN(KC_GEMV, macs, (double)gguf_byte_count((uint32_t)w.dtype, w.elements) + (double)M * (w.K + w.N) * 8,
            gemv_exact(d_a, w.K, M, w, d_c, w.N, shift, h->ws, st));
    } else {
        const double tc = h->plan.use_tc ? (double)M * (double)w.N * (double)h->plan.k_pad * tc::LA * h->plan.wlimbs : 0.0;
        run_k(ctx, KC_GEMM, macs, 0, st,
              [&] { return gemm_run(d_a, w.K, M, w, h->plan, d_c, w.N, shift, nullptr, 0, h->ws, st); }, tc);
    }
    CK(cudaGetLastError());
    return SLX_OK;
}

slx_status slx_matmul_q30(slx_ctx* ctx, const int64_t* a, int M, int K, int dtype, const uint8_t* w_raw, int64_t w_bytes,
                          int N, int half_composite, int scale_bits, int shift, int64_t* c) {
    if (!ctx || M <= 0 || K <= 0 || N <= 0 || !a || !w_raw || !c) return set_err(ctx, SLX_EINVAL, "bad arguments");
    CK(cudaSetDevice(ctx->device));
    cudaStream_t st = ctx->stream;
    int64_t need = gguf_byte_count((uint32_t)dtype, (int64_t)N * K);
    if (w_bytes < need) return set_err(ctx, SLX_EEOF, "weight buffer too small");
    int64_t *da = nullptr, *dc = nullptr;
    uint8_t* dw = nullptr;
    CK(cudaMalloc(&da, sizeof(int64_t) * M * K));
    CK(cudaMalloc(&dc, sizeof(int64_t) * M * N));
    CK(cudaMalloc(&dw, need));
    cudaMemsetAsync(ctx->d_flag, 0, sizeof(int), st);
    cudaMemcpyAsync(da, a, sizeof(int64_t) * M * K, cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(dw, w_raw, need, cudaMemcpyHostToDevice, st);
    int rc = slx_matmul_q30_device(ctx, da, M, K, dtype, dw, need, N, half_composite, scale_bits, shift, dc, st);
    if (!rc) {
        cudaMemcpyAsync(c, dc, sizeof(int64_t) * M * N, cudaMemcpyDeviceToHost, st);
        rc = check_flag(ctx, st);
    }
    cudaFree(da);
    cudaFree(dc);
    cudaFree(dw);
    return rc;
}

slx_status slx_attention(slx_ctx* ctx, const int64_t* q, const int64_t* k, const int64_t* v, int seq, int q_embd,
                         int kv_dim, int nh, int nkv, int scale_exp, int mode, int window, int64_t* out) {
    if (!ctx || !q || !k || !v || !out || seq <= 0 || nh <= 0 || nkv <= 0 || nh % nkv || q_embd % nh || kv_dim % nkv ||
        mode < 0 || mode > 2)
        return set_err(ctx, SLX_EINVAL, "bad arguments");
    const int hd = q_embd / nh;
    if (kv_dim / nkv != hd) return set_err(ctx, SLX_EINVAL, "q and kv head sizes differ");
    CK(cudaSetDevice(ctx->device));
    cudaStream_t st = ctx->stream;
    const size_t nq = (size_t)seq * q_embd, nk = (size_t)seq * kv_dim;
    int64_t *dq = nullptr, *dk = nullptr, *dv = nullptr, *dout = nullptr;
    void* ws = nullptr;
    const int abs_scale = scale_exp < 0 ? -scale_exp : scale_exp;
    const int sshift = 2 * abs_scale - 30;
    int64_t sq = isqrt64_host(hd);
    if (sq == 0) sq = 1;
    const bool tc = tc_enabled() && attention_tc_supported(seq, nh, nkv, hd);
    const size_t wsb = tc ? attention_tc_workspace(1, seq, nh, nkv, hd) : 0;
    int rc = SLX_OK;
    if (cudaMalloc(&dq, nq * 8) != cudaSuccess || cudaMalloc(&dk, nk * 8) != cudaSuccess ||
        cudaMalloc(&dv, nk * 8) != cudaSuccess || cudaMalloc(&dout, nq * 8) != cudaSuccess ||
        (wsb && cudaMalloc(&ws, wsb) != cudaSuccess)) {
        rc = set_err(ctx, SLX_EOOM, "device allocation failed");
    } else {
        cudaMemsetAsync(ctx->d_flag, 0, sizeof(int), st);
        cudaMemcpyAsync(dq, q, nq * 8, cudaMemcpyHostToDevice, st);
        cudaMemcpyAsync(dk, k, nk * 8, cudaMemcpyHostToDevice, st);
        cudaMemcpyAsync(dv, v, nk * 8, cudaMemcpyHostToDevice, st);
        int n = -1;
        if (tc) n = attention_tc(dq, q_embd, dk, kv_dim, dv, kv_dim, dout, q_embd, 1, seq, nh, nkv, hd, sshift, sq, mode,
                                 window, ws, ctx->d_flag, st);
        if (n < 0) n = attention(dq, q_embd, dk, kv_dim, dv, kv_dim, dout, q_embd, 1, seq, nh, nkv, hd, sshift, sq, mode,
                                 window, st);
        ctx->launches += n;
        cudaMemcpyAsync(out, dout, nq * 8, cudaMemcpyDeviceToHost, st);
        rc = check_flag(ctx, st);
    }
    cudaFree(dq); cudaFree(dk); cudaFree(dv); cudaFree(dout);
    if (ws) cudaFree(ws);
    return rc;
}

slx_status slx_profile_begin(slx_ctx* ctx) {
    if (!ctx) return SLX_EINVAL;
    for (auto& r : ctx->records) { ctx->event_pool.push_back(r.a); ctx->event_pool.push_back(r.b); }
    ctx->records.clear();
    ctx->prof = true;
    return SLX_OK;
}

slx_status slx_profile_end(slx_ctx* ctx, slx_kernel_stat* stats, int cap, int* n) {
    if (!ctx || !n) return SLX_EINVAL;
    ctx->prof = false;
    slx_kernel_stat acc[KC_COUNT];
    static_assert(sizeof(kKClassName) / sizeof(kKClassName[0]) == KC_COUNT, "kernel class names");
    std::memset(acc, 0, sizeof acc);
    for (int c = 0; c < KC_COUNT; c++) snprintf(acc[c].name, sizeof acc[c].name, "%s", kKClassName[c]);
    for (auto& r : ctx->records) {
        CK(cudaEventSynchronize(r.b));
        float ms = 0;
        CK(cudaEventElapsedTime(&ms, r.a, r.b));
        acc[r.cls].launches += r.launches;
        acc[r.cls].ms += ms;
        acc[r.cls].macs += r.macs;
        acc[r.cls].bytes += r.bytes;
        acc[r.cls].tc_macs += r.tc_macs;
        ctx->event_pool.push_back(r.a);
        ctx->event_pool.push_back(r.b);
    }
    ctx->records.clear();
    int k = 0;
    for (int c = 0; c < KC_COUNT; c++)
        if (acc[c].launches && k < cap && stats) stats[k++] = acc[c];
    *n = k;
    return SLX_OK;
}

slx_status slx_launch_count(slx_ctx* ctx, int64_t* launches) {
    if (!ctx || !launches) return SLX_EINVAL;
    *launches = ctx->launches;
    return SLX_OK;
}

// ---- lattice k-NN search ----------------------------------------------------------------------

struct slx_lattice {
    slx_ctx* ctx = nullptr;
    search::Lattice L;
    float zero_threshold = 0.001f;
    int64_t global_scale = 1000000000;
    tree::Tree tree;         // KD tree over the rows (built by slx_lattice_build_tree or loaded)
    bool has_tree = false;
};

slx_status slx_lattice_build_device(slx_ctx* ctx, const float* d_vectors, int64_t n, int dim, float zero_threshold,
                                    int64_t global_scale, int64_t id_base, void* stream, slx_lattice** out) {
    if (!ctx || !out) return set_err(ctx, SLX_EINVAL, "null argument");
    *out = nullptr;
    CK(cudaSetDevice(ctx->device));
    std::unique_ptr<slx_lattice> lat(new slx_lattice());
    lat->ctx = ctx;
    lat->zero_threshold = zero_threshold;
    lat->global_scale = global_scale;
    std::string err;
    cudaStream_t st = pick(ctx, stream);
    int rc = search::build(d_vectors, n, dim, zero_threshold, global_scale, id_base, lat->L, st, err);
    if (n > 0) ctx->launches += 2;
    if (rc) {
        search::release(lat->L);
        return set_err(ctx, rc, "%s", err.c_str());
    }
    ctx->refs.fetch_add(1);
    *out = lat.release();
    return SLX_OK;
}

slx_status slx_lattice_build(slx_ctx* ctx, const float* vectors, int64_t n, int dim, float zero_threshold,
                             int64_t global_scale, int64_t id_base, slx_lattice** out) {
    if (!ctx || !out || (n > 0 && !vectors) || n < 0 || dim < 1) return set_err(ctx, SLX_EINVAL, "bad arguments");
    CK(cudaSetDevice(ctx->device));
    float* d = nullptr;
    const size_t bytes = (size_t)n * dim * sizeof(float);
    if (bytes) {
        if (cudaMalloc(&d, bytes) != cudaSuccess) { cudaGetLastError(); return set_err(ctx, SLX_EOOM, "lattice input"); }
        cudaError_t e = cudaMemcpyAsync(d, vectors, bytes, cudaMemcpyHostToDevice, ctx->stream);
        if (e != cudaSuccess) { cudaFree(d); return set_err(ctx, SLX_ECUDA, "%s", cudaGetErrorString(e)); }
    }
    slx_status rc = slx_lattice_build_device(ctx, d, n, dim, zero_threshold, global_scale, id_base, nullptr, out);
    cudaStreamSynchronize(ctx->stream);
    cudaFree(d);
    return rc;
}

slx_status slx_lattice_free(slx_lattice* lat) {
    if (!lat) return SLX_EINVAL;
    slx_ctx* ctx = lat->ctx;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    tree::release(lat->tree);
    search::release(lat->L);
    delete lat;
    ctx_release(ctx);
    return SLX_OK;
}

// ---- KD tree and SLAT ------------------------------------------------------------------------

slx_status slx_lattice_build_tree(slx_lattice* lat, int leaf_threshold) {
    if (!lat) return SLX_EINVAL;
    slx_ctx* ctx = lat->ctx;
    if (leaf_threshold < 0) return set_err(ctx, SLX_EINVAL, "LeafThreshold must be >= 0");
    CK(cudaSetDevice(ctx->device));
    cudaStream_t st = ctx->stream;
    std::string err;
    int rc = 0;
    lat->has_tree = false;
    run_k(ctx, KC_SEARCH, (double)lat->L.n * lat->L.dim, 0, st, [&] {
        int64_t nl = 0;
        rc = tree::build(lat->L.vals, lat->L.n, lat->L.dim, leaf_threshold, lat->tree, st, err, &nl);
        return (int)nl;
    });
    if (rc) return set_err(ctx, rc, "%s", err.c_str());
    lat->has_tree = true;
    return SLX_OK;
}

slx_status slx_lattice_tree_info(slx_lattice* lat, int64_t* info, int n) {
    if (!lat || !info || n < 0) return SLX_EINVAL;
    if (!lat->has_tree) return set_err(lat->ctx, SLX_EINVAL, "the lattice has no tree (slx_lattice_build_tree)");
    const tree::Stats t = tree::stats(lat->tree);
    const int64_t v[5] = {t.nodes, t.branches, t.leaves, t.occupants, t.max_depth};
    for (int i = 0; i < n && i < 5; i++) info[i] = v[i];
    return SLX_OK;
}

slx_status slx_lattice_tree_export(slx_lattice* lat, int32_t* kind, int32_t* mask, int32_t* dim, int64_t* val,
                                   int64_t* start, int64_t* count, int32_t* perm) {
    if (!lat) return SLX_EINVAL;
    slx_ctx* ctx = lat->ctx;
    if (!lat->has_tree) return set_err(ctx, SLX_EINVAL, "the lattice has no tree (slx_lattice_build_tree)");
    const std::vector<int> order = tree::preorder(lat->tree);
    for (size_t i = 0; i < order.size(); i++) {
        const tree::Node& nd = lat->tree.nodes[order[i]];
        if (kind) kind[i] = nd.kind;
        if (mask) mask[i] = nd.mask;
        if (dim) dim[i] = nd.dim;
        if (val) val[i] = nd.val;
        if (start) start[i] = nd.start;
        if (count) count[i] = nd.count;
    }
    if (perm && lat->tree.n > 0) {
        CK(cudaSetDevice(ctx->device));
        CK(cudaMemcpyAsync(perm, lat->tree.perm, sizeof(int32_t) * lat->tree.n, cudaMemcpyDeviceToHost, ctx->stream));
        CK(cudaStreamSynchronize(ctx->stream));
    }
    return SLX_OK;
}

static slx_status lattice_save(slx_lattice* lat, tree::Sink& sink) {
    slx_ctx* ctx = lat->ctx;
    if (!lat->has_tree)
        return set_err(ctx, SLX_EINVAL, "Lattice must be frozen before serialization (slx_lattice_build_tree).");
    CK(cudaSetDevice(ctx->device));
    cudaStream_t st = ctx->stream;
    const int64_t n = lat->L.n;
    int32_t* d_pay = lat->L.payload;
    int32_t* tmp = nullptr;
    if (!d_pay && n > 0) {  // Int32 payloads: the row ids
        if (lat->L.id_base < INT32_MIN || lat->L.id_base + n - 1 > INT32_MAX)
            return set_err(ctx, SLX_EINVAL, "row ids id_base + row do not fit the Int32 payload");
        std::vector<int32_t> ids((size_t)n);
        for (int64_t i = 0; i < n; i++) ids[i] = (int32_t)(lat->L.id_base + i);
        CK(cudaMalloc(&tmp, sizeof(int32_t) * n));
        cudaMemcpyAsync(tmp, ids.data(), sizeof(int32_t) * n, cudaMemcpyHostToDevice, st);
        d_pay = tmp;
    }
    std::string err;
    int rc = 0;
    run_k(ctx, KC_SEARCH, 0, 0, st, [&] {
        int64_t nl = 0;
        rc = tree::save(lat->tree, lat->L.vals, lat->L.dim, d_pay, sink, st, err, &nl);
        return (int)nl;
    });
    cudaStreamSynchronize(st);
    cudaFree(tmp);
    if (rc) return set_err(ctx, rc, "%s", err.c_str());
    return SLX_OK;
}

slx_status slx_lattice_save_slat(slx_lattice* lat, const char* path) {
    if (!lat || !path) return lat ? set_err(lat->ctx, SLX_EINVAL, "null path") : SLX_EINVAL;
    FILE* f = fopen(path, "wb");
    if (!f) return set_err(lat->ctx, SLX_ENOTFOUND, "cannot open %s for writing", path);
    tree::Sink sink;
    sink.f = f;
    slx_status rc = lattice_save(lat, sink);
    if (fclose(f) != 0 && rc == SLX_OK) rc = set_err(lat->ctx, SLX_EINVAL, "write to %s failed", path);
    return rc;
}

slx_status slx_lattice_save_slat_mem(slx_lattice* lat, uint8_t* out, int64_t cap, int64_t* size) {
    if (!lat || !size || cap < 0) return lat ? set_err(lat->ctx, SLX_EINVAL, "bad arguments") : SLX_EINVAL;
    slx_ctx* ctx = lat->ctx;
    if (!lat->has_tree)
        return set_err(ctx, SLX_EINVAL, "Lattice must be frozen before serialization (slx_lattice_build_tree).");
    CK(cudaSetDevice(ctx->device));
    std::string err;
    int64_t need = 0, nl = 0;
    int rc = tree::slat_size(lat->tree, lat->L.vals, lat->L.dim, &need, ctx->stream, err, &nl);
    ctx->launches += nl;
    if (rc) return set_err(ctx, rc, "%s", err.c_str());
    *size = need;
    if (!out) return SLX_OK;
    if (cap < need)
        return set_err(ctx, SLX_EINVAL, "output buffer of %lld bytes, %lld needed", (long long)cap, (long long)need);
    tree::Sink sink;
    sink.mem = out;
    sink.cap = (size_t)cap;
    return lattice_save(lat, sink);
}

static slx_status lattice_load(slx_ctx* ctx, const uint8_t* bytes, int64_t n, float zero_threshold,
                               int64_t global_scale, slx_lattice** out) {
    tree::Loaded ld;
    std::string err;
    int rc = tree::parse(bytes, n, ld, err);
    if (rc) return set_err(ctx, rc, "%s", err.c_str());
    CK(cudaSetDevice(ctx->device));
    cudaStream_t st = ctx->stream;
    std::unique_ptr<slx_lattice> lat(new slx_lattice());
    lat->ctx = ctx;
    lat->zero_threshold = zero_threshold;
    lat->global_scale = global_scale;
    const int64_t rows = (int64_t)ld.payload.size();
    const int dim = ld.dim > 0 ? ld.dim : 1;
    int32_t* d_rows = nullptr;
    if (rows > 0) {
        if (cudaMalloc(&d_rows, sizeof(int32_t) * rows * dim) != cudaSuccess) {
            cudaGetLastError();
            return set_err(ctx, SLX_EOOM, "device allocation failed");
        }
        cudaMemcpyAsync(d_rows, ld.rows.data(), sizeof(int32_t) * rows * dim, cudaMemcpyHostToDevice, st);
    }
    rc = search::build_quantized(d_rows, rows, dim, 0, lat->L, st, err);
    cudaFree(d_rows);
    if (rc) {
        search::release(lat->L);
        return set_err(ctx, rc, "%s", err.c_str());
    }
    if (rows > 0) ctx->launches += 2;
    if (rows > 0 && cudaMalloc(&lat->L.payload, sizeof(int32_t) * rows) != cudaSuccess) {
        cudaGetLastError();
        search::release(lat->L);
        return set_err(ctx, SLX_EOOM, "device allocation failed");
    }
    if (rows > 0) cudaMemcpyAsync(lat->L.payload, ld.payload.data(), sizeof(int32_t) * rows, cudaMemcpyHostToDevice, st);
    // the tree as read; occupants are stored in file order, so leaf order is the identity
    lat->tree.nodes = std::move(ld.nodes);
    lat->tree.root = ld.root;
    lat->tree.n = rows;
    if (cudaMalloc(&lat->tree.perm, sizeof(int32_t) * (size_t)std::max<int64_t>(rows, 1)) != cudaSuccess) {
        cudaGetLastError();
        search::release(lat->L);
        return set_err(ctx, SLX_EOOM, "device allocation failed");
    }
    if (rows > 0) {
        std::vector<int32_t> id((size_t)rows);
        for (int64_t i = 0; i < rows; i++) id[i] = (int32_t)i;
        cudaMemcpyAsync(lat->tree.perm, id.data(), sizeof(int32_t) * rows, cudaMemcpyHostToDevice, st);
    }
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        tree::release(lat->tree);
        search::release(lat->L);
        return set_err(ctx, SLX_ECUDA, "%s", cudaGetErrorString(e));
    }
    lat->has_tree = true;
    ctx->refs.fetch_add(1);
    *out = lat.release();
    return SLX_OK;
}

slx_status slx_lattice_load_slat_mem(slx_ctx* ctx, const uint8_t* bytes, int64_t n, float zero_threshold,
                                     int64_t global_scale, slx_lattice** out) {
    if (!ctx || !out || n < 0 || (n > 0 && !bytes)) return set_err(ctx, SLX_EINVAL, "bad arguments");
    *out = nullptr;
    return lattice_load(ctx, bytes, n, zero_threshold, global_scale, out);
}

slx_status slx_lattice_load_slat(slx_ctx* ctx, const char* path, float zero_threshold, int64_t global_scale,
                                 slx_lattice** out) {
    if (!ctx || !out || !path) return set_err(ctx, SLX_EINVAL, "bad arguments");
    *out = nullptr;
    FILE* f = fopen(path, "rb");
    if (!f) return set_err(ctx, SLX_ENOTFOUND, "Could not find file '%s'.", path);
    std::vector<uint8_t> bytes;
    uint8_t chunk[1 << 16];
    size_t got;
    while ((got = fread(chunk, 1, sizeof chunk, f)) > 0) bytes.insert(bytes.end(), chunk, chunk + got);
    fclose(f);
    return lattice_load(ctx, bytes.data(), (int64_t)bytes.size(), zero_threshold, global_scale, out);
}

slx_status slx_lattice_info(slx_lattice* lat, int64_t* info, int n) {
    if (!lat || !info || n < 0) return SLX_EINVAL;
    const int64_t v[3] = {lat->L.n, lat->L.dim, lat->L.id_base};
    for (int i = 0; i < n && i < 3; i++) info[i] = v[i];
    return SLX_OK;
}

slx_status slx_lattice_query_knn_l2_device(slx_lattice* lat, const float* d_queries, int nq, int k, int flags,
                                           int64_t* d_ids, uint64_t* d_dist, int* n_exact, void* stream) {
    if (!lat) return SLX_EINVAL;
    slx_ctx* ctx = lat->ctx;
    CK(cudaSetDevice(ctx->device));
    cudaStream_t st = pick(ctx, stream);
    std::string err;
    int rc = 0;
    run_k(ctx, KC_SEARCH, 2.0 * nq * (double)lat->L.n * lat->L.dim, 0, st, [&] {
        int64_t nl = 0;
        rc = search::query(lat->L, d_queries, nq, k, lat->zero_threshold, lat->global_scale,
                           (flags & SLX_KNN_EXACT) != 0, d_ids, d_dist, n_exact, st, err, &nl);
        return (int)nl;
    });
    if (rc) return set_err(ctx, rc, "%s", err.c_str());
    return SLX_OK;
}

slx_status slx_lattice_query_knn_l2(slx_lattice* lat, const float* queries, int nq, int k, int flags, int64_t* ids,
                                    uint64_t* dist, int* n_exact) {
    if (!lat) return SLX_EINVAL;
    slx_ctx* ctx = lat->ctx;
    if (nq < 0 || k < 0 || (nq > 0 && k > 0 && (!queries || !ids || !dist)))
        return set_err(ctx, SLX_EINVAL, "bad arguments");
    if (n_exact) *n_exact = 0;
    if (nq == 0 || k == 0) return SLX_OK;
    CK(cudaSetDevice(ctx->device));
    const size_t qb = (size_t)nq * lat->L.dim * sizeof(float), ob = (size_t)nq * k * 8;
    void* buf = nullptr;
    if (cudaMalloc(&buf, qb + 2 * ob + 512) != cudaSuccess) { cudaGetLastError(); return set_err(ctx, SLX_EOOM, "query buffers"); }
    float* dq = (float*)buf;
    int64_t* di = (int64_t*)((char*)buf + ((qb + 255) & ~(size_t)255));
    uint64_t* dd = (uint64_t*)((char*)di + ((ob + 255) & ~(size_t)255));
    cudaMemcpyAsync(dq, queries, qb, cudaMemcpyHostToDevice, ctx->stream);
    slx_status rc = slx_lattice_query_knn_l2_device(lat, dq, nq, k, flags, di, dd, n_exact, nullptr);
    if (rc == SLX_OK) {
        cudaMemcpyAsync(ids, di, ob, cudaMemcpyDeviceToHost, ctx->stream);
        cudaMemcpyAsync(dist, dd, ob, cudaMemcpyDeviceToHost, ctx->stream);
        cudaError_t e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) rc = set_err(ctx, SLX_ECUDA, "%s", cudaGetErrorString(e));
    } else {
        cudaStreamSynchronize(ctx->stream);
    }
    cudaFree(buf);
    return rc;
}

slx_status slx_knn_merge_device(slx_ctx* ctx, const int64_t* d_ids, const uint64_t* d_dist, int parts, int nq, int k,
                                int64_t* d_out_ids, uint64_t* d_out_dist, void* stream) {
    if (!ctx || parts < 1 || parts > 64 || nq < 0 || k < 0) return set_err(ctx, SLX_EINVAL, "bad arguments");
    if (nq == 0 || k == 0) return SLX_OK;
    if (!d_ids || !d_dist || !d_out_ids || !d_out_dist) return set_err(ctx, SLX_EINVAL, "null buffer");
    CK(cudaSetDevice(ctx->device));
    cudaStream_t st = pick(ctx, stream);
    run_k(ctx, KC_SEARCH, 0, 0, st, [&] {
        search::merge_parts(d_ids, d_dist, parts, nq, k, d_out_ids, d_out_dist, st);
        return 1;
    });
    CK(cudaGetLastError());
    return SLX_OK;
}

}  // extern "C"
