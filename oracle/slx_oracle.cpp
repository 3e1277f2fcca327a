// slx_oracle.cpp -- CPU restatement of SparseLattice's quantized integer transformer forward.
//
// TEST INFRASTRUCTURE ONLY. This file is the parity oracle and the timed CPU baseline. Only the
// tests, the smoke check and the bench's CPU-baseline / reference legs load it; the product
// library (spatialdb_b200) never links or calls it.
//
// It restates, function by function, the C# reference (damiant3/SpatialDb, project SparseLattice):
//   Gguf/GgufReader.cs, Gguf/GgufDequantizer.cs, Gguf/GgufTensorInfo.cs, Gguf/GgufTypes.cs,
//   Math/IntegerMatMul.cs, Math/IntegerTranscendentals.cs, Math/IntegerLayerNorm.cs,
//   Math/IntegerAttention.cs, Math/IntegerFFN.cs, Gguf/IntegerTransformerSource*.cs,
//   Gguf/IntegerCausalSource*.cs, Gguf/IntegerGemmaSource*.cs, Lattice/VocabLattice.cs,
//   and for the lattice k-NN search Math/EmbeddingAdapter.cs, Math/SparseVector.cs,
//   Lattice/EmbeddingLattice.cs (KnnHeap), Lattice/RecallEvaluator.cs.
// Each function names the file:line it follows. C# semantics reproduced here:
//   * Int128 and long arithmetic is unchecked (wraps); accumulation is done in unsigned __int128
//     so wrap-around is defined in C++ too.
//   * `/` on integers truncates toward zero, `>>` on signed values floors.
//   * (long)double truncates; NaN or out-of-range gives long.MinValue (x64 cvttsd2si, .NET 8).
//   * (Half)float rounds to nearest even; float arithmetic is never FMA-contracted
//     (built with -ffp-contract=off).
//
// Parity pinning: the reference cannot run in this environment (C#, no .NET runtime), so this
// restatement is pinned by the reference's own known-answer unit tests, ported in tests/.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>
#include <algorithm>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef __int128 i128;
typedef unsigned __int128 u128;

extern "C" {
enum {
    SLXO_OK = 0,
    SLXO_EINVAL = 1,       // ArgumentException / bad shape
    SLXO_EFORMAT = 2,      // InvalidDataException (magic, version, value type)
    SLXO_ENOTFOUND = 3,    // KeyNotFoundException / FileNotFoundException
    SLXO_EUNSUPPORTED = 4, // NotSupportedException (dtype, architecture)
    SLXO_EEOF = 5,         // EndOfStreamException
    SLXO_ERANGE = 6,       // IndexOutOfRangeException (MXFP4 nibble 15, RoPE row past the table)
};
}

// ------------------------------------------------------------------------------------------
// C# numeric helpers
// ------------------------------------------------------------------------------------------
static inline int64_t cs_d2l(double v) {
    // (long)double: truncation toward zero; NaN / out of range -> long.MinValue (x64 .NET 8).
    if (v >= -9223372036854775808.0 && v < 9223372036854775808.0) return (int64_t)v;
    return INT64_MIN;
}
static inline int64_t wrap_add(int64_t a, int64_t b) { return (int64_t)((uint64_t)a + (uint64_t)b); }
static inline int64_t wrap_sub(int64_t a, int64_t b) { return (int64_t)((uint64_t)a - (uint64_t)b); }
static inline int64_t wrap_mul(int64_t a, int64_t b) { return (int64_t)((uint64_t)a * (uint64_t)b); }
static inline int64_t lo64(i128 v) { return (int64_t)(uint64_t)(u128)v; }
// Int128 >> n with C#'s shift-count masking (n & 127); arithmetic (floor) for signed values.
static inline i128 sar128(i128 v, int n) { return v >> (n & 127); }
// C# long / long (truncating). long.MinValue / -1 throws in C#; never reached on these paths.
static inline int64_t cs_div64(int64_t a, int64_t b) {
    if (b == -1) return wrap_sub(0, a);
    return a / b;
}

// GgufDequantizer.HalfToFloat (GgufDequantizer.cs:327-328): exact binary16 -> binary32.
static float half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {  // subnormal: renormalise
            int e = -1;
            do { man <<= 1; e++; } while ((man & 0x400) == 0);
            man &= 0x3ff;
            bits = sign | (uint32_t)(127 - 15 - e) << 23 | (man << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13) | (man ? 0x400000u : 0u);
    } else {
        bits = sign | ((exp + 112) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

// (Half)float, IEEE round-to-nearest-even (IntegerCausalSource.Loading.cs:218-225 ReadAsHalf,
// IntegerGemmaSource.Loading.cs:178-184 ToHalf).
static uint16_t float_to_half(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) {  // inf / nan
        if (ax == 0x7f800000u) return sign | 0x7c00;
        return (uint16_t)(sign | 0x7c00 | 0x200 | ((ax >> 13) & 0x3ff));
    }
    if (ax >= 0x477ff000u) return sign | 0x7c00;  // >= 65520 rounds to infinity
    if (ax < 0x38800000u) {                        // below 2^-14: half subnormal or zero
        uint32_t e = ax >> 23;
        if (e == 0) return sign;                   // float subnormal -> 0
        uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        int s = 126 - (int)e;                       // value / 2^-24 = m >> s
        if (s > 24) return sign;
        uint32_t r = m >> s;
        uint32_t rem = m & ((1u << s) - 1);
        uint32_t halfway = 1u << (s - 1);
        if (rem > halfway || (rem == halfway && (r & 1))) r++;
        return (uint16_t)(sign | r);
    }
    uint32_t e = ax >> 23;
    uint32_t man = ax & 0x7fffffu;
    uint32_t h = ((e - 112) << 10) | (man >> 13);
    uint32_t rem = man & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) h++;
    return (uint16_t)(sign | h);
}

static float bits_to_float(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }

// Q30 value of every half bit pattern: (long)((float)h * 2^30) (IntegerMatMul.cs:262).
static int64_t g_half_q30[65536];
static bool g_half_q30_ready = false;
static void init_half_q30(int scale_bits) {
    // Built per scale; the models here always use scale_bits=30, other scales recompute.
    static int built_for = -1;
    if (g_half_q30_ready && built_for == scale_bits) return;
    double scale = (double)(1LL << scale_bits);
    for (int i = 0; i < 65536; i++) g_half_q30[i] = cs_d2l((double)half_to_float((uint16_t)i) * scale);
    built_for = scale_bits;
    g_half_q30_ready = true;
}

// ------------------------------------------------------------------------------------------
// GGUF container (GgufReader.cs:54-130, GgufTensorInfo.cs:27-48, GgufTypes.cs:4-38)
// ------------------------------------------------------------------------------------------
enum GgufType { F32 = 0, F16 = 1, Q4_0 = 2, Q4_1 = 3, Q5_0 = 6, Q5_1 = 7, Q8_0 = 8, Q2_K = 10,
                Q3_K = 11, Q4_K = 12, Q5_K = 13, Q6_K = 14, Q8_K = 15, BF16 = 30, MXFP4 = 39 };

struct GValue {
    uint32_t type = 0;
    int64_t i = 0;       // signed view of integer types
    uint64_t u = 0;      // unsigned view
    double f = 0;
    std::string s;
    std::vector<GValue> arr;
};

struct GTensor {
    std::string name;
    std::vector<int> shape;
    uint32_t dtype = 0;
    int64_t offset = 0;
    int64_t elements = 0;
    int64_t bytes = 0;
};

// GgufTensorInfo.ComputeByteCount (GgufTensorInfo.cs:27-48)
static int64_t gguf_byte_count(uint32_t dtype, int64_t e) {
    switch (dtype) {
        case F32: return e * 4;
        case F16: return e * 2;
        case BF16: return e * 2;
        case Q8_0: return (e / 32) * (2 + 32);
        case Q4_0: return (e / 32) * (2 + 16);
        case Q4_1: return (e / 32) * (2 + 2 + 16);
        case Q5_0: return (e / 32) * (2 + 4 + 16);
        case Q5_1: return (e / 32) * (2 + 2 + 4 + 16);
        case Q2_K: return (e / 256) * (2 + 2 + 256 / 16 + 256 / 4);
        case Q3_K: return (e / 256) * (2 + 256 / 8 + 256 / 4 + 12);
        case Q4_K: return (e / 256) * (2 + 2 + 12 + 256 / 2);
        case Q5_K: return (e / 256) * (2 + 2 + 12 + 256 / 2 + 256 / 8);
        case Q6_K: return (e / 256) * (2 + 256 / 2 + 256 / 4 + 256 / 16);
        case Q8_K: return (e / 256) * (4 + 256 + 16 * 2);
        case MXFP4: return (e / 32) * 17;
        default: return e * 4;
    }
}

struct Gguf {
    FILE* fp = nullptr;
    uint32_t version = 0;
    int64_t data_offset = 0;
    std::map<std::string, GValue> meta;
    std::vector<GTensor> tensors;
    std::map<std::string, size_t> index;
    std::string arch;
    int embd = 0, ctx = 0, heads = 0, layers = 0, ff = 0;
    int n_tokens = 0, bos = 0, eos = 0, unk = 0;
    ~Gguf() { if (fp) fclose(fp); }
};

struct Rd {
    FILE* fp;
    bool eof = false;
    void raw(void* p, size_t n) { if (!eof && fread(p, 1, n, fp) != n) eof = true; if (eof) memset(p, 0, n); }
    uint8_t u8() { uint8_t v; raw(&v, 1); return v; }
    uint16_t u16() { uint16_t v; raw(&v, 2); return v; }
    uint32_t u32() { uint32_t v; raw(&v, 4); return v; }
    uint64_t u64() { uint64_t v; raw(&v, 8); return v; }
    std::string str() {  // ReadGgufString (GgufReader.cs:206-212)
        uint64_t n = u64();
        if (eof || n == 0) return "";
        if (n > (1ull << 31)) { eof = true; return ""; }
        std::string s(n, '\0');
        raw(&s[0], n);
        return s;
    }
};

// ReadValue / ReadArrayValue (GgufReader.cs:214-243). Returns false on an unknown type.
static bool read_value(Rd& r, uint32_t t, GValue& v) {
    v.type = t;
    switch (t) {
        case 0: v.u = r.u8(); v.i = (int64_t)v.u; break;
        case 1: v.i = (int8_t)r.u8(); v.u = (uint64_t)v.i; break;
        case 2: v.u = r.u16(); v.i = (int64_t)v.u; break;
        case 3: v.i = (int16_t)r.u16(); v.u = (uint64_t)v.i; break;
        case 4: v.u = r.u32(); v.i = (int64_t)v.u; break;
        case 5: v.i = (int32_t)r.u32(); v.u = (uint64_t)v.i; break;
        case 6: { uint32_t b = r.u32(); v.f = bits_to_float(b); break; }
        case 7: v.u = r.u8() != 0; v.i = (int64_t)v.u; break;
        case 8: v.s = r.str(); break;
        case 9: {
            uint32_t et = r.u32();
            uint64_t n = r.u64();
            if (r.eof) return true;
            if (n > (1ull << 32)) { r.eof = true; return true; }
            v.arr.resize(n);
            for (uint64_t k = 0; k < n && !r.eof; k++)
                if (!read_value(r, et, v.arr[k])) return false;
            break;
        }
        case 10: v.u = r.u64(); v.i = (int64_t)v.u; break;
        case 11: v.i = (int64_t)r.u64(); v.u = (uint64_t)v.i; break;
        case 12: { uint64_t b = r.u64(); memcpy(&v.f, &b, 8); break; }
        default: return false;
    }
    return true;
}

// GgufReader.GetInt (GgufReader.cs:252-263): Int32/UInt32/Int64/UInt64 else 0.
static int meta_int(const Gguf& g, const std::string& k) {
    auto it = g.meta.find(k);
    if (it == g.meta.end()) return 0;
    const GValue& v = it->second;
    switch (v.type) {
        case 5: return (int)v.i;
        case 4: return (int)(uint32_t)v.u;
        case 11: return (int)v.i;
        case 10: return (int)v.u;
        default: return 0;
    }
}
// IntegerCausalSource.GetInt (IntegerCausalSource.Loading.cs:246-255): Int32/UInt32 else default.
static int meta_int_i32(const Gguf& g, const std::string& k, int def) {
    auto it = g.meta.find(k);
    if (it == g.meta.end()) return def;
    if (it->second.type == 5) return (int)it->second.i;
    if (it->second.type == 4) return (int)(uint32_t)it->second.u;
    return def;
}
// *Source.GetFloat (IntegerTransformerSource.Loading.cs:156-165): Float32/Float64 else default.
static float meta_float(const Gguf& g, const std::string& k, float def) {
    auto it = g.meta.find(k);
    if (it == g.meta.end()) return def;
    if (it->second.type == 6) return (float)it->second.f;
    if (it->second.type == 12) return (float)it->second.f;
    return def;
}

// GgufReader ctor (GgufReader.cs:54-130).
static Gguf* gguf_open(const char* path, int* status) {
    FILE* fp = fopen(path, "rb");
    if (!fp) { *status = SLXO_ENOTFOUND; return nullptr; }
    std::unique_ptr<Gguf> g(new Gguf());
    g->fp = fp;
    Rd r{fp};
    uint32_t magic = r.u32();
    if (r.eof) { *status = SLXO_EEOF; return nullptr; }
    if (magic != 0x46554747u) { *status = SLXO_EFORMAT; return nullptr; }
    g->version = r.u32();
    if (r.eof) { *status = SLXO_EEOF; return nullptr; }
    if (g->version != 2 && g->version != 3) { *status = SLXO_EFORMAT; return nullptr; }
    uint64_t n_tensors = r.u64();
    uint64_t n_meta = r.u64();
    for (uint64_t i = 0; i < n_meta && !r.eof; i++) {
        std::string key = r.str();
        uint32_t t = r.u32();
        GValue v;
        if (!read_value(r, t, v)) { *status = SLXO_EFORMAT; return nullptr; }
        g->meta[key] = std::move(v);
    }
    for (uint64_t i = 0; i < n_tensors && !r.eof; i++) {
        GTensor t;
        t.name = r.str();
        uint32_t nd = r.u32();
        if (nd > 64) { *status = SLXO_EFORMAT; return nullptr; }
        t.shape.resize(nd);
        int64_t e = 1;
        for (uint32_t d = 0; d < nd; d++) { t.shape[d] = (int)r.u64(); e *= t.shape[d]; }
        t.dtype = r.u32();
        t.offset = (int64_t)r.u64();
        t.elements = e;
        t.bytes = gguf_byte_count(t.dtype, e);
        g->tensors.push_back(t);
    }
    if (r.eof) { *status = SLXO_EEOF; return nullptr; }
    long pos = ftell(fp);
    g->data_offset = (pos + 31L) & ~31L;
    for (size_t i = 0; i < g->tensors.size(); i++) g->index[g->tensors[i].name] = i;
    auto it = g->meta.find("general.architecture");
    g->arch = (it != g->meta.end() && it->second.type == 8) ? it->second.s : "";
    const std::string& a = g->arch;
    g->embd = meta_int(*g, a + ".embedding_length");
    g->ctx = meta_int(*g, a + ".context_length");
    g->heads = meta_int(*g, a + ".attention.head_count");
    g->layers = meta_int(*g, a + ".block_count");
    g->ff = meta_int(*g, a + ".feed_forward_length");
    auto tk = g->meta.find("tokenizer.ggml.tokens");
    g->n_tokens = (tk != g->meta.end() && tk->second.type == 9) ? (int)tk->second.arr.size() : 0;
    g->bos = meta_int(*g, "tokenizer.ggml.bos_token_id");
    g->eos = meta_int(*g, "tokenizer.ggml.eos_token_id");
    g->unk = meta_int(*g, "tokenizer.ggml.unknown_token_id");
    *status = SLXO_OK;
    return g.release();
}

// ------------------------------------------------------------------------------------------
// Dequantizers (GgufDequantizer.cs)
// ------------------------------------------------------------------------------------------
static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// Returns the number of raw bytes the dtype's reader consumes for n output floats.
static int64_t dequant_bytes_needed(uint32_t dtype, int64_t n) {
    switch (dtype) {
        case F32: return n * 4;
        case F16: case BF16: return n * 2;
        case Q8_0: return (n / 32) * 34;
        case Q4_0: return (n / 32) * 18;
        case MXFP4: return (n / 32) * 17;
        case Q2_K: return (n / 256) * 84;
        case Q3_K: return (n / 256) * 110;
        case Q4_K: return (n / 256) * 144;
        case Q5_K: return (n / 256) * 176;
        case Q6_K: return (n / 256) * 210;
        case Q8_K: return (n / 256) * 292;
        default: return -1;
    }
}

// UnpackQ4KScales (GgufDequantizer.cs:345-357)
static void unpack_q4k_scales(const uint8_t* raw, uint8_t* sc, uint8_t* m) {
    for (int j = 0; j < 4; j++) { sc[j] = raw[j] & 63; m[j] = raw[j + 4] & 63; }
    for (int j = 4; j < 8; j++) {
        sc[j] = (uint8_t)((raw[j + 4] & 0x0F) | ((raw[j - 4] >> 6) << 4));
        m[j] = (uint8_t)((raw[j + 4] >> 4) | ((raw[j] >> 6) << 4));
    }
}

// The MXFP4 table as the reference declares it (GgufDequantizer.cs:91-95): the missing comma in
// "-4.0f -6.0f" folds the last two entries into -10.0f, leaving 15 entries.
static const float k_mxfp4[15] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                                  -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -10.0f};

// Dispatch of GgufReader.ReadTensorF32 (GgufReader.cs:172-201) over an in-memory byte buffer.
static int dequantize(uint32_t dtype, const uint8_t* buf, int64_t len, float* out, int64_t n) {
    int64_t need = dequant_bytes_needed(dtype, n);
    if (need < 0) return SLXO_EUNSUPPORTED;
    if (len < need) return SLXO_EEOF;
    switch (dtype) {
        case F32:  // ReadF32 (:7-17)
            memcpy(out, buf, (size_t)n * 4);
            return SLXO_OK;
        case F16:  // ReadF16 (:19-29)
            for (int64_t i = 0; i < n; i++) out[i] = half_to_float(rd16(buf + 2 * i));
            return SLXO_OK;
        case BF16:  // DequantizeBF16 (:78-89)
            for (int64_t i = 0; i < n; i++) out[i] = bits_to_float((uint32_t)rd16(buf + 2 * i) << 16);
            return SLXO_OK;
        case Q8_0: {  // DequantizeQ8_0 (:31-49)
            int64_t blocks = n / 32, o = 0, in = 0;
            for (int64_t b = 0; b < blocks; b++) {
                float scale = half_to_float(rd16(buf + in));
                in += 2;
                for (int j = 0; j < 32; j++) out[o++] = scale * (float)(int8_t)buf[in++];
            }
            return SLXO_OK;
        }
        case Q4_0: {  // DequantizeQ4_0 (:51-76): element 2j = low nibble, 2j+1 = high nibble
            int64_t blocks = n / 32, o = 0, in = 0;
            for (int64_t b = 0; b < blocks; b++) {
                float scale = half_to_float(rd16(buf + in));
                in += 2;
                for (int j = 0; j < 16; j++) {
                    uint8_t raw = buf[in++];
                    int lo = (raw & 0x0F) - 8;
                    int hi = (raw >> 4) - 8;
                    out[o++] = scale * (float)lo;
                    out[o++] = scale * (float)hi;
                }
            }
            return SLXO_OK;
        }
        case MXFP4: {  // DequantizeMXFP4 (:97-123)
            int64_t blocks = n / 32, o = 0, in = 0;
            for (int64_t b = 0; b < blocks; b++) {
                uint8_t e8m0 = buf[in++];
                float shared = (e8m0 == 0) ? 0.0f : ldexpf(1.0f, (int)e8m0 - 127);
                for (int j = 0; j < 16; j++) {
                    uint8_t raw = buf[in++];
                    int lo = raw & 0x0F, hi = (raw >> 4) & 0x0F;
                    if (lo >= 15) return SLXO_ERANGE;
                    out[o++] = k_mxfp4[lo] * shared;
                    if (hi >= 15) return SLXO_ERANGE;
                    out[o++] = k_mxfp4[hi] * shared;
                }
            }
            return SLXO_OK;
        }
        case Q2_K: {  // DequantizeQ2K (:125-156)
            int64_t sbs = n / 256, o = 0, in = 0;
            for (int64_t s = 0; s < sbs; s++) {
                float d = half_to_float(rd16(buf + in));
                float dmin = half_to_float(rd16(buf + in + 2));
                const uint8_t* scales = buf + in + 4;
                const uint8_t* qs = buf + in + 20;
                in += 84;
                for (int j = 0; j < 256; j++) {
                    uint8_t sb = scales[j / 16];
                    int sc = sb & 0x0F, m = sb >> 4;
                    int q = (qs[j / 4] >> ((j % 4) * 2)) & 3;
                    out[o++] = d * (float)sc * (float)q - dmin * (float)m;
                }
            }
            return SLXO_OK;
        }
        case Q3_K: {  // DequantizeQ3K (:158-199)
            int64_t sbs = n / 256, o = 0, in = 0;
            int scales[16];
            for (int64_t s = 0; s < sbs; s++) {
                const uint8_t* hmask = buf + in;
                const uint8_t* qs = buf + in + 32;
                const uint8_t* sc = buf + in + 96;
                float d = half_to_float(rd16(buf + in + 108));
                in += 110;
                for (int j = 0; j < 16; j++) {
                    int low4 = (j < 8) ? (sc[j] & 0x0F) : (sc[j - 8] >> 4);
                    int high2 = (sc[8 + j / 4] >> (2 * (j % 4))) & 3;
                    scales[j] = (low4 | (high2 << 4)) - 32;
                }
                for (int j = 0; j < 256; j++) {
                    int qlow = (qs[j / 4] >> ((j % 4) * 2)) & 3;
                    int hbit = (hmask[j / 8] >> (j % 8)) & 1;
                    int q = qlow | (hbit << 2);
                    out[o++] = d * (float)scales[j / 16] * (float)(q - 4);
                }
            }
            return SLXO_OK;
        }
        case Q4_K:    // DequantizeQ4K (:201-232)
        case Q5_K: {  // DequantizeQ5K (:234-268)
            bool q5 = dtype == Q5_K;
            int64_t sbs = n / 256, o = 0, in = 0;
            uint8_t sc[8], m[8];
            for (int64_t s = 0; s < sbs; s++) {
                float d = half_to_float(rd16(buf + in));
                float dmin = half_to_float(rd16(buf + in + 2));
                unpack_q4k_scales(buf + in + 4, sc, m);
                const uint8_t* qh = buf + in + 16;
                const uint8_t* qs = buf + in + (q5 ? 48 : 16);
                in += q5 ? 176 : 144;
                for (int j = 0; j < 256; j++) {
                    int sub = j / 32;
                    int qb = qs[j / 2];
                    int q = (j % 2 == 0) ? (qb & 0x0F) : (qb >> 4);
                    if (q5) q |= ((qh[j / 8] >> (j % 8)) & 1) << 4;
                    out[o++] = d * (float)sc[sub] * (float)q - dmin * (float)m[sub];
                }
            }
            return SLXO_OK;
        }
        case Q6_K: {  // DequantizeQ6K (:270-303)
            int64_t sbs = n / 256, o = 0, in = 0;
            for (int64_t s = 0; s < sbs; s++) {
                const uint8_t* ql = buf + in;
                const uint8_t* qh = buf + in + 128;
                const uint8_t* scales = buf + in + 192;
                float d = half_to_float(rd16(buf + in + 208));
                in += 210;
                for (int j = 0; j < 256; j++) {
                    int8_t sc = (int8_t)scales[j / 16];
                    int qb = ql[j / 2];
                    int qlow = (j % 2 == 0) ? (qb & 0x0F) : (qb >> 4);
                    int qhigh = (qh[j / 4] >> ((j % 4) * 2)) & 3;
                    int q = qlow | (qhigh << 4);
                    out[o++] = d * (float)sc * (float)(q - 32);
                }
            }
            return SLXO_OK;
        }
        case Q8_K: {  // DequantizeQ8K (:305-325)
            int64_t sbs = n / 256, o = 0, in = 0;
            for (int64_t s = 0; s < sbs; s++) {
                float d;
                memcpy(&d, buf + in, 4);
                const uint8_t* qs = buf + in + 4;
                in += 292;
                for (int j = 0; j < 256; j++) out[o++] = d * (float)(int8_t)qs[j];
            }
            return SLXO_OK;
        }
    }
    return SLXO_EUNSUPPORTED;
}

// GgufReader.ReadTensorF32 (GgufReader.cs:141-145,172-201).
static int gguf_read_f32(Gguf* g, const std::string& name, std::vector<float>& out) {
    auto it = g->index.find(name);
    if (it == g->index.end()) return SLXO_ENOTFOUND;
    const GTensor& t = g->tensors[it->second];
    int64_t need = dequant_bytes_needed(t.dtype, t.elements);
    if (need < 0) return SLXO_EUNSUPPORTED;
    out.assign((size_t)t.elements, 0.0f);
    std::vector<uint8_t> buf((size_t)need);
    if (fseek(g->fp, g->data_offset + t.offset, SEEK_SET) != 0) return SLXO_EEOF;
    size_t got = need ? fread(buf.data(), 1, (size_t)need, g->fp) : 0;
    if ((int64_t)got != need) return SLXO_EEOF;
    return dequantize(t.dtype, buf.data(), need, out.data(), t.elements);
}

// ------------------------------------------------------------------------------------------
// IntegerMatMul (Math/IntegerMatMul.cs)
// ------------------------------------------------------------------------------------------
// DotInt128 (IntegerMatMul.cs:209-229); accumulation wraps mod 2^128 like C#'s unchecked Int128.
static inline i128 dot_i128(const int64_t* a, const int64_t* b, int n) {
    u128 acc = 0;
    for (int i = 0; i < n; i++) acc += (u128)((i128)a[i] * (i128)b[i]);
    return (i128)acc;
}
static inline int64_t shift_result(i128 acc, int shift) {
    return shift > 0 ? lo64(sar128(acc, shift)) : lo64(acc);
}

// MatMul(long[] a, ..., long[] w, colsB, resultShift) (IntegerMatMul.cs:37-76); W[col*colsA+k].
static void matmul_long(const int64_t* a, int rows, int cols, const int64_t* w, int colsB, int shift,
                        int64_t* c) {
#pragma omp parallel for schedule(static) if (colsB >= 256 && cols >= 256)
    for (int col = 0; col < colsB; col++) {
        const int64_t* wc = w + (int64_t)col * cols;
        for (int row = 0; row < rows; row++)
            c[(int64_t)row * colsB + col] = shift_result(dot_i128(a + (int64_t)row * cols, wc, cols), shift);
    }
}

// MatMul(long[] a, ..., Half[] w, colsB, scaleBits, resultShift) (IntegerMatMul.cs:166-205) with
// DotInt128Mixed(Half) (:255-275): each weight is (long)((float)h * 2^scaleBits).
static void matmul_half(const int64_t* a, int rows, int cols, const uint16_t* w, int colsB, int scale_bits,
                        int shift, int64_t* c) {
    init_half_q30(scale_bits);
#pragma omp parallel if (colsB >= 256 && cols >= 256)
    {
        std::vector<int64_t> wq((size_t)cols);
#pragma omp for schedule(static)
        for (int col = 0; col < colsB; col++) {
            const uint16_t* wc = w + (int64_t)col * cols;
            for (int k = 0; k < cols; k++) wq[k] = g_half_q30[wc[k]];
            for (int row = 0; row < rows; row++)
                c[(int64_t)row * colsB + col] = shift_result(dot_i128(a + (int64_t)row * cols, wq.data(), cols), shift);
        }
    }
}

// MatMul(long[] a, ..., float[] w, colsB, scaleBits, resultShift) (IntegerMatMul.cs:121-160) with
// DotInt128Mixed(float) (:232-252).
static void matmul_float(const int64_t* a, int rows, int cols, const float* w, int colsB, int scale_bits,
                         int shift, int64_t* c) {
    double scale = (double)(1LL << scale_bits);
#pragma omp parallel if (colsB >= 256 && cols >= 256)
    {
        std::vector<int64_t> wq((size_t)cols);
#pragma omp for schedule(static)
        for (int col = 0; col < colsB; col++) {
            const float* wc = w + (int64_t)col * cols;
            for (int k = 0; k < cols; k++) wq[k] = cs_d2l((double)wc[k] * scale);
            for (int row = 0; row < rows; row++)
                c[(int64_t)row * colsB + col] = shift_result(dot_i128(a + (int64_t)row * cols, wq.data(), cols), shift);
        }
    }
}

// QuantizeFromFloat (IntegerMatMul.cs:297-304)
static void quantize_from_float(const float* src, int64_t n, int bits, int64_t* out) {
    double scale = (double)(1LL << bits);
    for (int64_t i = 0; i < n; i++) out[i] = cs_d2l((double)src[i] * scale);
}

// AddInPlace (IntegerMatMul.cs:284-288), unchecked long addition.
static void add_in_place(int64_t* dst, const int64_t* src, int64_t n) {
    for (int64_t i = 0; i < n; i++) dst[i] = wrap_add(dst[i], src[i]);
}

// ------------------------------------------------------------------------------------------
// IntegerTranscendentals (Math/IntegerTranscendentals.cs)
// ------------------------------------------------------------------------------------------
static inline int64_t fixed_from_double(double v, int frac) { return cs_d2l(v * (double)(1LL << frac)); }

// FixedExp (IntegerTranscendentals.cs:13-47)
static int64_t fixed_exp(int64_t x, int frac) {
    int64_t ln2 = fixed_from_double(0.6931471805599453, frac);
    if (ln2 == 0) ln2 = 1;
    int64_t k = x >= 0 ? x / ln2 : wrap_sub(0, cs_div64(wrap_sub(wrap_add(wrap_sub(0, x), ln2), 1), ln2));
    int64_t r = wrap_sub(x, wrap_mul(k, ln2));
    if (k > 62) return INT64_MAX;
    if (k < -(frac + 10)) return 0;
    int64_t one = 1LL << frac;
    int64_t term = one, sum = one;
    for (int n = 1; n <= 14; n++) {
        i128 num = (i128)term * (i128)r;
        i128 den = (i128)n << frac;
        term = lo64(num / den);
        sum = wrap_add(sum, term);
        if (term == 0 && n > 4) break;
    }
    if (k >= 0) {
        if (k >= 63 || sum > (INT64_MAX >> k)) return INT64_MAX;
        return (int64_t)((uint64_t)sum << k);
    }
    int sh = (int)(-k);
    if (sh >= 63) return 0;
    return sum >> sh;
}

// FixedSigmoid (IntegerTranscendentals.cs:49-63)
static int64_t fixed_sigmoid(int64_t x, int frac) {
    int64_t one = 1LL << frac;
    int64_t thr = 20LL * one;
    if (x > thr) return one;
    if (x < -thr) return 0;
    int64_t e = fixed_exp(wrap_sub(0, x), frac);
    int64_t den = wrap_add(one, e);
    if (den == 0) return one;
    return lo64(((i128)one * one) / (i128)den);
}

// FixedSiLU (IntegerTranscendentals.cs:65-69)
static int64_t fixed_silu(int64_t x, int frac) {
    int64_t sig = fixed_sigmoid(x, frac);
    return lo64(sar128((i128)x * sig, frac));
}

// FixedSoftmax (IntegerTranscendentals.cs:71-97)
static void fixed_softmax(int64_t* s, int len, int frac) {
    int64_t one = 1LL << frac;
    int64_t mx = s[0];
    for (int i = 1; i < len; i++) if (s[i] > mx) mx = s[i];
    u128 sum = 0;
    for (int i = 0; i < len; i++) {
        int64_t e = fixed_exp(wrap_sub(s[i], mx), frac);
        s[i] = e;
        sum += (u128)(i128)e;
    }
    if (sum == 0) {
        int64_t uni = one / len;
        for (int i = 0; i < len; i++) s[i] = uni;
        return;
    }
    i128 ssum = (i128)sum;
    for (int i = 0; i < len; i++) s[i] = lo64(((i128)s[i] * one) / ssum);
}

// ------------------------------------------------------------------------------------------
// IntegerLayerNorm (Math/IntegerLayerNorm.cs)
// ------------------------------------------------------------------------------------------
// ISqrt64 (IntegerLayerNorm.cs:130-149): floor(sqrt(value)) for value > 0, 0 otherwise. The reference's double seed plus Newton
// and fix-up loops return the exact floor, which is unique, so any exact method agrees.
static int64_t isqrt64(int64_t v) {
    if (v <= 0) return 0;
    if (v == 1) return 1;
    int64_t x = (int64_t)std::sqrt((double)v);
    if (x <= 0) x = 1;
    while (x > 0 && (i128)x * x > v) x--;
    while ((i128)(x + 1) * (x + 1) <= v) x++;
    return x;
}

// ISqrt128 (IntegerLayerNorm.cs:99-122): exact floor sqrt, returned as (long). Values at or
// above 2^126 make the reference's (x+1)^2 fix-up overflow Int128; such variances need
// |x - mean| near 2^63 and are outside any Q30 activation range.
static int64_t isqrt128(i128 v) {
    if (v <= 0) return 0;
    if (v <= (i128)INT64_MAX) return isqrt64((int64_t)v);
    u128 uv = (u128)v;
    u128 x = (u128)std::sqrt((long double)uv);
    if (x == 0) x = 1;
    for (int it = 0; it < 8; it++) {
        u128 nx = (x + uv / x) >> 1;
        if (nx >= x) break;
        x = nx;
    }
    while (x * x > uv) x--;
    while ((x + 1) * (x + 1) <= uv) x++;
    return (int64_t)(uint64_t)x;
}

// NormalizeRow (IntegerLayerNorm.cs:21-57): mean, variance, isqrt, scale, bias.
static void layernorm_row(int64_t* x, int embd, const int64_t* w, const int64_t* b) {
    u128 sum = 0;
    for (int d = 0; d < embd; d++) sum += (u128)(i128)x[d];
    int64_t mean = lo64((i128)sum / embd);
    u128 ss = 0;
    for (int d = 0; d < embd; d++) {
        int64_t delta = wrap_sub(x[d], mean);
        ss += (u128)((i128)delta * delta);
    }
    i128 var = (i128)ss / embd;
    if (var <= 0) {
        for (int d = 0; d < embd; d++) x[d] = b[d];
        return;
    }
    int64_t isq = isqrt128(var);
    if (isq == 0) isq = 1;
    for (int d = 0; d < embd; d++) {
        int64_t delta = wrap_sub(x[d], mean);
        i128 prod = (i128)delta * w[d];
        x[d] = wrap_add(lo64(prod / isq), b[d]);
    }
}

// ApplyInPlace (IntegerLayerNorm.cs:13-18)
static void layernorm(int64_t* x, int seq, int embd, const int64_t* w, const int64_t* b) {
    for (int t = 0; t < seq; t++) layernorm_row(x + (int64_t)t * embd, embd, w, b);
}

// RmsNormRow (IntegerLayerNorm.cs:71-93)
static void rmsnorm_row(int64_t* x, int embd, const int64_t* w) {
    u128 ss = 0;
    for (int d = 0; d < embd; d++) ss += (u128)((i128)x[d] * x[d]);
    i128 ms = (i128)ss / embd;
    if (ms <= 0) return;
    int64_t rms = isqrt128(ms);
    if (rms == 0) rms = 1;
    for (int d = 0; d < embd; d++) x[d] = lo64(((i128)x[d] * w[d]) / rms);
}

// RmsNormInPlace (IntegerLayerNorm.cs:63-68)
static void rmsnorm(int64_t* x, int seq, int embd, const int64_t* w) {
    for (int t = 0; t < seq; t++) rmsnorm_row(x + (int64_t)t * embd, embd, w);
}

// RmsNormPerHead (IntegerCausalSource.Forward.cs:123-130, IntegerGemmaSource.Forward.cs:88-95)
static void rmsnorm_per_head(int64_t* x, int seq, int nh, int hd, const int64_t* w) {
    for (int t = 0; t < seq; t++)
        for (int h = 0; h < nh; h++) rmsnorm_row(x + ((int64_t)t * nh + h) * hd, hd, w);
}

// ------------------------------------------------------------------------------------------
// IntegerAttention (Math/IntegerAttention.cs)
// ------------------------------------------------------------------------------------------
struct RoPE {
    int max_seq = 0, half = 0, frac = 30;
    std::vector<int64_t> cos, sin;
};

// IntegerRoPECache ctor (IntegerAttention.cs:14-32)
static void rope_build(RoPE& c, int max_seq, int head_dim, float base, int frac) {
    c.max_seq = max_seq;
    c.half = head_dim / 2;
    c.frac = frac;
    c.cos.assign((size_t)max_seq * c.half, 0);
    c.sin.assign((size_t)max_seq * c.half, 0);
    for (int t = 0; t < max_seq; t++)
        for (int i = 0; i < c.half; i++) {
            double theta = std::pow((double)base, -2.0 * i / head_dim);
            double angle = t * theta;
            c.cos[(size_t)t * c.half + i] = fixed_from_double(std::cos(angle), frac);
            c.sin[(size_t)t * c.half + i] = fixed_from_double(std::sin(angle), frac);
        }
}

// ApplyRoPE (IntegerAttention.cs:35-58): NeoX rotate-half pairs (i, i + halfDim).
static int apply_rope(int64_t* x, int seq, int embd, int nh, const RoPE& c) {
    int hd = embd / nh, half = hd / 2, fb = c.frac;
    if (seq > c.max_seq) return SLXO_ERANGE;
    for (int t = 0; t < seq; t++) {
        const int64_t* cr = c.cos.data() + (size_t)t * c.half;
        const int64_t* sr = c.sin.data() + (size_t)t * c.half;
        for (int h = 0; h < nh; h++) {
            int64_t* hb = x + (int64_t)t * embd + (int64_t)h * hd;
            for (int i = 0; i < half; i++) {
                int64_t co = cr[i], si = sr[i];
                int64_t x0 = hb[i], x1 = hb[i + half];
                hb[i] = lo64(sar128((i128)((u128)((i128)x0 * co) - (u128)((i128)x1 * si)), fb));
                hb[i + half] = lo64(sar128((i128)((u128)((i128)x0 * si) + (u128)((i128)x1 * co)), fb));
            }
        }
    }
    return SLXO_OK;
}

// One attention head (NonCausalHeadAttention :165-202, CausalHeadAttention :246-289,
// SlidingWindowHeadAttention :333-377; MultiHeadAttention :60-109 is the nKv == nHeads case).
// mode 0 = non-causal, 1 = causal (mask -2^(frac-1)), 2 = causal + sliding window.
static void head_attention(const int64_t* q, const int64_t* k, const int64_t* v, int64_t* out, int seq,
                           int q_embd, int kv_dim, int h, int hd, int kv_hd, int heads_per_kv, int score_shift,
                           int64_t sqrt_hd, int64_t mask, int mode, int window, int frac) {
    int kvh = h / heads_per_kv;
    int qoff = h * hd, kvoff = kvh * kv_hd;
    std::vector<int64_t> sc((size_t)seq * seq);
    for (int t = 0; t < seq; t++) {
        const int64_t* qb = q + (int64_t)t * q_embd + qoff;
        int ws = std::max(0, t - window + 1);
        for (int s = 0; s < seq; s++) {
            if ((mode >= 1 && s > t) || (mode == 2 && s < ws)) {
                sc[(size_t)t * seq + s] = mask;
                continue;
            }
            i128 raw = dot_i128(qb, k + (int64_t)s * kv_dim + kvoff, hd);
            sc[(size_t)t * seq + s] = cs_div64(lo64(sar128(raw, score_shift)), sqrt_hd);
        }
    }
    for (int t = 0; t < seq; t++) fixed_softmax(sc.data() + (size_t)t * seq, seq, frac);
    for (int t = 0; t < seq; t++) {
        int64_t* ob = out + (int64_t)t * q_embd + qoff;
        for (int s = 0; s < seq; s++) {
            int64_t wgt = sc[(size_t)t * seq + s];
            const int64_t* vb = v + (int64_t)s * kv_dim + kvoff;
            for (int d = 0; d < hd; d++) ob[d] = wrap_add(ob[d], lo64(sar128((i128)wgt * vb[d], frac)));
        }
    }
}

// GroupedQueryAttention (:125-163), CausalGroupedQueryAttention (:205-244),
// SlidingWindowCausalGQA (:293-331), MultiHeadAttention (:60-109).
static void gqa(const int64_t* q, const int64_t* k, const int64_t* v, int seq, int q_embd, int kv_dim, int nh,
                int nkv, int scale_exp, int frac, int mode, int window, int64_t* out) {
    int hd = q_embd / nh, kv_hd = kv_dim / nkv, hpk = nh / nkv;
    memset(out, 0, sizeof(int64_t) * (size_t)seq * q_embd);
    int abs_scale = scale_exp < 0 ? -scale_exp : scale_exp;
    int score_shift = 2 * abs_scale - frac;
    int64_t sq = isqrt64(hd);
    if (sq == 0) sq = 1;
    int64_t mask = -(1LL << (frac - 1));
#pragma omp parallel for schedule(dynamic) if (nh >= 4)
    for (int h = 0; h < nh; h++)
        head_attention(q, k, v, out, seq, q_embd, kv_dim, h, hd, kv_hd, hpk, score_shift, sq, mask, mode, window, frac);
}

// ------------------------------------------------------------------------------------------
// IntegerFFN (Math/IntegerFFN.cs)
// ------------------------------------------------------------------------------------------
static void silu_gate(const int64_t* gate, int64_t* up, int64_t n, int frac) {
    for (int64_t i = 0; i < n; i++) up[i] = lo64(sar128((i128)fixed_silu(gate[i], frac) * up[i], frac));
}

// Apply(long[] ...) (IntegerFFN.cs:70-100)
static void ffn_long(const int64_t* x, int seq, int embd, const int64_t* wg, const int64_t* wu, const int64_t* wd,
                     int nff, int shift, int frac, int64_t* out) {
    std::vector<int64_t> gate((size_t)seq * nff), up((size_t)seq * nff);
    matmul_long(x, seq, embd, wg, nff, shift, gate.data());
    matmul_long(x, seq, embd, wu, nff, shift, up.data());
    silu_gate(gate.data(), up.data(), (int64_t)seq * nff, frac);
    matmul_long(up.data(), seq, nff, wd, embd, shift, out);
}

// Apply(long[] ..., Half[] ...) (IntegerFFN.cs:6-36)
static void ffn_half(const int64_t* x, int seq, int embd, const uint16_t* wg, const uint16_t* wu, const uint16_t* wd,
                     int nff, int scale_bits, int frac, int64_t* out) {
    std::vector<int64_t> gate((size_t)seq * nff), up((size_t)seq * nff);
    matmul_half(x, seq, embd, wg, nff, scale_bits, scale_bits, gate.data());
    matmul_half(x, seq, embd, wu, nff, scale_bits, scale_bits, up.data());
    silu_gate(gate.data(), up.data(), (int64_t)seq * nff, frac);
    matmul_half(up.data(), seq, nff, wd, embd, scale_bits, scale_bits, out);
}

// ------------------------------------------------------------------------------------------
// IntegerTransformerSource: nomic-bert / bert encoder (Gguf/IntegerTransformerSource*.cs)
// ------------------------------------------------------------------------------------------
struct EncLayer { std::vector<int64_t> qkv, o, anw, anb, up, gate, down, lnw, lnb; };
struct Encoder {
    int embd = 0, heads = 0, layers = 0, ff = 0, scale_bits = 30, unk = 0;
    float rope_base = 10000.0f;
    std::vector<int64_t> tok, tt, enw, enb;
    std::vector<EncLayer> L;
    RoPE rope;
    int64_t vocab_rows = 0;
};

static int read_q(Gguf* g, const std::string& name, int bits, std::vector<int64_t>& out) {
    std::vector<float> f;
    int st = gguf_read_f32(g, name, f);
    if (st) return st;
    out.resize(f.size());
    quantize_from_float(f.data(), (int64_t)f.size(), bits, out.data());
    return SLXO_OK;
}

// Load / LoadFromReader (IntegerTransformerSource.Loading.cs:47-151)
static Encoder* encoder_load(const char* path, int scale_bits, int* status) {
    std::unique_ptr<Gguf> g(gguf_open(path, status));
    if (!g) return nullptr;
    std::string a = g->arch;
    std::string al = a;
    std::transform(al.begin(), al.end(), al.begin(), ::tolower);
    if (al != "nomic-bert" && al != "bert") { *status = SLXO_EUNSUPPORTED; return nullptr; }
    std::unique_ptr<Encoder> e(new Encoder());
    e->embd = g->embd; e->heads = g->heads; e->layers = g->layers; e->ff = g->ff;
    e->scale_bits = scale_bits;
    e->rope_base = meta_float(*g, a + ".rope.freq_base", 10000.0f);
    int st;
    if ((st = read_q(g.get(), "token_embd.weight", scale_bits, e->tok))) { *status = st; return nullptr; }
    std::vector<float> tt;
    if ((st = gguf_read_f32(g.get(), "token_types.weight", tt))) { *status = st; return nullptr; }
    if ((int64_t)tt.size() < e->embd) { *status = SLXO_EINVAL; return nullptr; }
    e->tt.resize(e->embd);
    quantize_from_float(tt.data(), e->embd, scale_bits, e->tt.data());
    if ((st = read_q(g.get(), "token_embd_norm.weight", scale_bits, e->enw))) { *status = st; return nullptr; }
    if ((st = read_q(g.get(), "token_embd_norm.bias", scale_bits, e->enb))) { *status = st; return nullptr; }
    e->L.resize(e->layers);
    for (int i = 0; i < e->layers; i++) {
        std::string p = "blk." + std::to_string(i);
        EncLayer& l = e->L[i];
        const char* names[9] = {".attn_qkv.weight", ".attn_output.weight", ".attn_output_norm.weight",
                                ".attn_output_norm.bias", ".ffn_up.weight", ".ffn_gate.weight", ".ffn_down.weight",
                                ".layer_output_norm.weight", ".layer_output_norm.bias"};
        std::vector<int64_t>* dst[9] = {&l.qkv, &l.o, &l.anw, &l.anb, &l.up, &l.gate, &l.down, &l.lnw, &l.lnb};
        for (int j = 0; j < 9; j++)
            if ((st = read_q(g.get(), p + names[j], scale_bits, *dst[j]))) { *status = st; return nullptr; }
    }
    // WordPieceTokenizer.FromGguf (WordPieceTokenizer.cs:23-30) rejects an empty vocabulary.
    if (g->n_tokens == 0) { *status = SLXO_EINVAL; return nullptr; }
    e->unk = g->unk;
    e->vocab_rows = (int64_t)e->tok.size();
    // GetRoPECache (IntegerTransformerSource.Forward.cs:101-108): 512 rows.
    rope_build(e->rope, 512, e->embd / e->heads, e->rope_base, 30);
    *status = SLXO_OK;
    return e.release();
}

// BuildEmbeddings (IntegerTransformerSource.Forward.cs:7-26): UNK row when the id is out of range.
static void encoder_embed(const Encoder& e, const int32_t* ids, int T, int64_t* x) {
    int d = e.embd;
    for (int t = 0; t < T; t++) {
        int64_t src = (int64_t)ids[t] * d;
        if (ids[t] < 0 || src + d > (int64_t)e.tok.size()) src = (int64_t)e.unk * d;
        for (int j = 0; j < d; j++) x[(int64_t)t * d + j] = wrap_add(e.tok[src + j], e.tt[j]);
    }
}

// ApplyTransformerBlock (IntegerTransformerSource.Forward.cs:28-67)
static int encoder_block(const Encoder& e, const EncLayer& l, int64_t* x, int T) {
    int d = e.embd, sb = e.scale_bits;
    int64_t tot = (int64_t)T * d;
    std::vector<int64_t> res(x, x + tot), qkv((size_t)T * 3 * d), q(tot), k(tot), v(tot);
    matmul_long(x, T, d, l.qkv.data(), 3 * d, sb, qkv.data());
    for (int t = 0; t < T; t++) {  // SplitQkv (IntegerAttention.cs:111-121)
        memcpy(&q[(size_t)t * d], &qkv[(size_t)t * 3 * d], sizeof(int64_t) * d);
        memcpy(&k[(size_t)t * d], &qkv[(size_t)t * 3 * d + d], sizeof(int64_t) * d);
        memcpy(&v[(size_t)t * d], &qkv[(size_t)t * 3 * d + 2 * d], sizeof(int64_t) * d);
    }
    int st;
    if ((st = apply_rope(q.data(), T, d, e.heads, e.rope))) return st;
    if ((st = apply_rope(k.data(), T, d, e.heads, e.rope))) return st;
    std::vector<int64_t> att(tot), proj(tot);
    gqa(q.data(), k.data(), v.data(), T, d, d, e.heads, e.heads, -sb, 30, 0, 0, att.data());
    matmul_long(att.data(), T, d, l.o.data(), d, sb, proj.data());
    add_in_place(proj.data(), res.data(), tot);
    layernorm(proj.data(), T, d, l.anw.data(), l.anb.data());
    std::vector<int64_t> rf(proj), fo(tot);
    ffn_long(proj.data(), T, d, l.gate.data(), l.up.data(), l.down.data(), e.ff, sb, 30, fo.data());
    add_in_place(fo.data(), rf.data(), tot);
    layernorm(fo.data(), T, d, l.lnw.data(), l.lnb.data());
    memcpy(x, fo.data(), sizeof(int64_t) * tot);
    return SLXO_OK;
}

// Forward up to the last layer's output (IntegerTransformerSource.cs:65-78 without MeanPool).
static int encoder_hidden(const Encoder& e, const int32_t* ids, int T, int n_layers, int64_t* x) {
    encoder_embed(e, ids, T, x);
    layernorm(x, T, e.embd, e.enw.data(), e.enb.data());
    int nl = n_layers < 0 ? e.layers : std::min(n_layers, e.layers);
    for (int i = 0; i < nl; i++) {
        int st = encoder_block(e, e.L[i], x, T);
        if (st) return st;
    }
    return SLXO_OK;
}

// MeanPool (IntegerTransformerSource.Forward.cs:69-87)
static void mean_pool(const int64_t* x, int T, int d, int64_t* pooled) {
    for (int j = 0; j < d; j++) {
        if (T == 0) { pooled[j] = 0; continue; }
        u128 s = 0;
        for (int t = 0; t < T; t++) s += (u128)(i128)x[(int64_t)t * d + j];
        pooled[j] = lo64((i128)s / T);
    }
}

// ForwardFloat + L2Normalize (IntegerTransformerSource.cs:52-62, .Forward.cs:89-99): sequential
// fp32 without FMA contraction.
static void to_float_l2(const int64_t* v, int d, int scale_bits, float* out) {
    double scale = std::pow(2.0, -scale_bits);
    for (int j = 0; j < d; j++) out[j] = (float)((double)v[j] * scale);
    float norm = 0.0f;
    for (int j = 0; j < d; j++) norm += out[j] * out[j];
    norm = std::sqrt(norm);
    if (norm < 1e-10f) return;
    float inv = 1.0f / norm;
    for (int j = 0; j < d; j++) out[j] *= inv;
}

// ------------------------------------------------------------------------------------------
// IntegerCausalSource / IntegerGemmaSource (Gguf/IntegerCausalSource*.cs, IntegerGemmaSource*.cs)
// ------------------------------------------------------------------------------------------
struct GemmaLayer {
    std::vector<int64_t> attn_norm, qn, kn, post_attn, ffn_norm, post_ffw;
    std::vector<uint16_t> q, k, v, o, gate, up, down;
};
struct Causal {
    int embd = 0, heads = 0, kv_heads = 0, head_dim = 0, q_dim = 0, kv_dim = 0, ff = 0, layers = 0;
    int vocab = 0, scale_bits = 30, sliding = 0, global_interval = 0, unk = 0, eos = 0;
    float rope_base = 10000.0f, rope_base_global = 10000.0f;
    std::vector<uint16_t> tok;
    std::vector<int64_t> tok_q30;  // IntegerGemmaSource keeps token rows as Q30 long
    std::vector<int64_t> out_norm;
    std::vector<GemmaLayer> L;
    RoPE rope_local, rope_global;
    bool causal = true;  // false: IntegerGemmaSource encoder semantics
    mutable std::vector<int64_t> vocab_q;  // the VocabLattice's quantized rows, built on first use
};

static int read_half(Gguf* g, const std::string& name, std::vector<uint16_t>& out) {
    std::vector<float> f;
    int st = gguf_read_f32(g, name, f);
    if (st) return st;
    out.resize(f.size());
    for (size_t i = 0; i < f.size(); i++) out[i] = float_to_half(f[i]);
    return SLXO_OK;
}

// LoadFromReader (IntegerCausalSource.Loading.cs:74-195): norms as Q30 long, projections as Half,
// missing q/k/post norms replaced by ones (MakeOnesWeight :227-233).
// With gemma_encoder set it follows IntegerGemmaSource.LoadFromReader
// (IntegerGemmaSource.Loading.cs:80-157): token rows as Q30 long, every norm tensor required.
static Causal* causal_load(const char* path, int scale_bits, int* status, bool gemma_encoder) {
    std::unique_ptr<Gguf> g(gguf_open(path, status));
    if (!g) return nullptr;
    std::string a = g->arch, al = a;
    std::transform(al.begin(), al.end(), al.begin(), ::tolower);
    if (al.rfind("gemma", 0) != 0) { *status = SLXO_EUNSUPPORTED; return nullptr; }
    std::unique_ptr<Causal> c(new Causal());
    c->embd = g->embd; c->heads = g->heads; c->layers = g->layers; c->ff = g->ff;
    c->kv_heads = meta_int_i32(*g, a + ".attention.head_count_kv", c->heads);
    c->head_dim = meta_int_i32(*g, a + ".attention.key_length", c->heads ? c->embd / c->heads : 0);
    c->rope_base = meta_float(*g, a + ".rope.freq_base", 10000.0f);
    c->vocab = g->n_tokens;
    c->sliding = meta_int_i32(*g, a + ".attention.sliding_window", 0);
    c->global_interval = c->sliding > 0 ? 6 : 0;
    c->rope_base_global = c->sliding > 0 ? 1000000.0f : c->rope_base;
    c->q_dim = c->heads * c->head_dim;
    c->kv_dim = c->kv_heads * c->head_dim;
    c->scale_bits = scale_bits;
    c->causal = !gemma_encoder;
    int st;
    if (gemma_encoder) {
        if ((st = read_q(g.get(), "token_embd.weight", scale_bits, c->tok_q30))) { *status = st; return nullptr; }
    } else {
        if ((st = read_half(g.get(), "token_embd.weight", c->tok))) { *status = st; return nullptr; }
    }
    if ((st = read_q(g.get(), "output_norm.weight", scale_bits, c->out_norm))) { *status = st; return nullptr; }
    auto ones = [&](int n) { return std::vector<int64_t>((size_t)n, 1LL << scale_bits); };
    c->L.resize(c->layers);
    for (int i = 0; i < c->layers; i++) {
        std::string p = "blk." + std::to_string(i);
        GemmaLayer& l = c->L[i];
        if ((st = read_q(g.get(), p + ".attn_norm.weight", scale_bits, l.attn_norm))) { *status = st; return nullptr; }
        if ((st = read_half(g.get(), p + ".attn_q.weight", l.q))) { *status = st; return nullptr; }
        if ((st = read_half(g.get(), p + ".attn_k.weight", l.k))) { *status = st; return nullptr; }
        if ((st = read_half(g.get(), p + ".attn_v.weight", l.v))) { *status = st; return nullptr; }
        bool req = gemma_encoder;
        if (req || g->index.count(p + ".attn_q_norm.weight")) { if ((st = read_q(g.get(), p + ".attn_q_norm.weight", scale_bits, l.qn))) { *status = st; return nullptr; } }
        else l.qn = ones(c->heads * c->head_dim);
        if (req || g->index.count(p + ".attn_k_norm.weight")) { if ((st = read_q(g.get(), p + ".attn_k_norm.weight", scale_bits, l.kn))) { *status = st; return nullptr; } }
        else l.kn = ones(c->kv_heads * c->head_dim);
        if ((st = read_half(g.get(), p + ".attn_output.weight", l.o))) { *status = st; return nullptr; }
        if (req || g->index.count(p + ".post_attention_norm.weight")) { if ((st = read_q(g.get(), p + ".post_attention_norm.weight", scale_bits, l.post_attn))) { *status = st; return nullptr; } }
        else l.post_attn = ones(c->embd);
        if ((st = read_q(g.get(), p + ".ffn_norm.weight", scale_bits, l.ffn_norm))) { *status = st; return nullptr; }
        if ((st = read_half(g.get(), p + ".ffn_gate.weight", l.gate))) { *status = st; return nullptr; }
        if ((st = read_half(g.get(), p + ".ffn_up.weight", l.up))) { *status = st; return nullptr; }
        if ((st = read_half(g.get(), p + ".ffn_down.weight", l.down))) { *status = st; return nullptr; }
        if (req || g->index.count(p + ".post_ffw_norm.weight")) { if ((st = read_q(g.get(), p + ".post_ffw_norm.weight", scale_bits, l.post_ffw))) { *status = st; return nullptr; } }
        else l.post_ffw = ones(c->embd);
    }
    c->unk = g->unk;
    c->eos = g->eos;
    // GetRoPECacheLocal / GetRoPECacheGlobal (IntegerCausalSource.Forward.cs:132-146): 2048 rows.
    rope_build(c->rope_local, 2048, c->head_dim, c->rope_base, 30);
    rope_build(c->rope_global, 2048, c->head_dim, c->rope_base_global, 30);
    *status = SLXO_OK;
    return c.release();
}

// BuildEmbeddings (IntegerCausalSource.Forward.cs:7-31): (long)((float)Half * 2^30) * ISqrt64(d).
// IntegerGemmaSource.BuildEmbeddings (IntegerGemmaSource.Forward.cs:7-30) copies Q30 long rows
// before the same ISqrt64(d) scaling.
static void causal_embed(const Causal& c, const int32_t* ids, int T, int64_t* x) {
    init_half_q30(c.scale_bits);
    int d = c.embd;
    int64_t sq = isqrt64(d);
    int64_t rows = c.causal ? (int64_t)c.tok.size() : (int64_t)c.tok_q30.size();
    for (int t = 0; t < T; t++) {
        int64_t src = (int64_t)ids[t] * d;
        if (ids[t] < 0 || src + d > rows) src = (int64_t)c.unk * d;
        for (int j = 0; j < d; j++) {
            int64_t e = c.causal ? g_half_q30[c.tok[src + j]] : c.tok_q30[src + j];
            x[(int64_t)t * d + j] = lo64((i128)e * sq);
        }
    }
}

// IsGlobalLayer (IntegerCausalSource.Forward.cs:38-43)
static bool is_global(const Causal& c, int li) {
    if (c.global_interval <= 0) return true;
    return ((li + 1) % c.global_interval) == 0;
}

// ApplyCausalBlock (IntegerCausalSource.Forward.cs:45-114); with causal == false it is
// ApplyGemmaBlock (IntegerGemmaSource.Forward.cs:32-75).
static int causal_block(const Causal& c, const GemmaLayer& l, int64_t* x, int T, bool global) {
    int d = c.embd, sb = c.scale_bits;
    int64_t tot = (int64_t)T * d;
    std::vector<int64_t> res(x, x + tot);
    rmsnorm(x, T, d, l.attn_norm.data());
    std::vector<int64_t> q((size_t)T * c.q_dim), k((size_t)T * c.kv_dim), v((size_t)T * c.kv_dim);
    matmul_half(x, T, d, l.q.data(), c.q_dim, sb, sb, q.data());
    matmul_half(x, T, d, l.k.data(), c.kv_dim, sb, sb, k.data());
    matmul_half(x, T, d, l.v.data(), c.kv_dim, sb, sb, v.data());
    rmsnorm_per_head(q.data(), T, c.heads, c.head_dim, l.qn.data());
    rmsnorm_per_head(k.data(), T, c.kv_heads, c.head_dim, l.kn.data());
    const RoPE& rope = (global || !c.causal) ? c.rope_global : c.rope_local;
    int st;
    if ((st = apply_rope(q.data(), T, c.q_dim, c.heads, rope))) return st;
    if ((st = apply_rope(k.data(), T, c.kv_dim, c.kv_heads, rope))) return st;
    std::vector<int64_t> att((size_t)T * c.q_dim), proj(tot);
    int mode = !c.causal ? 0 : ((global || c.sliding <= 0) ? 1 : 2);
    gqa(q.data(), k.data(), v.data(), T, c.q_dim, c.kv_dim, c.heads, c.kv_heads, -sb, 30, mode, c.sliding, att.data());
    matmul_half(att.data(), T, c.q_dim, l.o.data(), d, sb, sb, proj.data());
    rmsnorm(proj.data(), T, d, l.post_attn.data());
    add_in_place(proj.data(), res.data(), tot);
    memcpy(res.data(), proj.data(), sizeof(int64_t) * tot);
    rmsnorm(proj.data(), T, d, l.ffn_norm.data());
    std::vector<int64_t> fo(tot);
    ffn_half(proj.data(), T, d, l.gate.data(), l.up.data(), l.down.data(), c.ff, sb, 30, fo.data());
    rmsnorm(fo.data(), T, d, l.post_ffw.data());
    add_in_place(fo.data(), res.data(), tot);
    memcpy(x, fo.data(), sizeof(int64_t) * tot);
    return SLXO_OK;
}

// ForwardCausal (IntegerCausalSource.cs:128-147) up to n_layers, then output norm if all ran.
static int causal_hidden(const Causal& c, const int32_t* ids, int T, int n_layers, bool final_norm, int64_t* x) {
    causal_embed(c, ids, T, x);
    int nl = n_layers < 0 ? c.layers : std::min(n_layers, c.layers);
    for (int i = 0; i < nl; i++) {
        int st = causal_block(c, c.L[i], x, T, is_global(c, i));
        if (st) return st;
    }
    if (final_norm) rmsnorm(x, T, c.embd, c.out_norm.data());
    return SLXO_OK;
}

// VocabLattice.ArgmaxBruteForce(float[], Half[], vocab, dims) (Lattice/VocabLattice.cs:103-126):
// sequential fp32 multiply-then-add, strict '>' so the first max wins.
static int argmax_half(const float* h, const uint16_t* E, int64_t n_elems, int vocab, int dims) {
    int best = 0;
    float best_score = -INFINITY;
    int64_t max_vocab = n_elems / dims;
    if (vocab > max_vocab) vocab = (int)max_vocab;
    for (int tid = 0; tid < vocab; tid++) {
        const uint16_t* row = E + (int64_t)tid * dims;
        float dot = 0.0f;
        for (int j = 0; j < dims; j++) {
            float p = h[j] * half_to_float(row[j]);
            dot = dot + p;
        }
        if (dot > best_score) { best_score = dot; best = tid; }
    }
    return best;
}

// ForwardCausalFloat (IntegerCausalSource.cs:114-122) + PredictNextToken (:149-161, lattice off).
static int causal_next(const Causal& c, const int32_t* ids, int T, int32_t* next, int64_t* last_out) {
    std::vector<int64_t> x((size_t)T * c.embd);
    int st = causal_hidden(c, ids, T, -1, true, x.data());
    if (st) return st;
    const int64_t* last = x.data() + (size_t)(T - 1) * c.embd;
    if (last_out) memcpy(last_out, last, sizeof(int64_t) * c.embd);
    std::vector<float> h(c.embd);
    double scale = std::pow(2.0, -c.scale_bits);
    for (int j = 0; j < c.embd; j++) h[j] = (float)((double)last[j] * scale);
    *next = argmax_half(h.data(), c.tok.data(), (int64_t)c.tok.size(), c.vocab, c.embd);
    return SLXO_OK;
}

// ==========================================================================================
// C ABI for the Python test harness (ctypes)
// ==========================================================================================

// ------------------------------------------------------------------------------------------
// Lattice k-NN search (embed + search)
// ------------------------------------------------------------------------------------------
// EmbeddingAdapter.QuantizeDense (Math/EmbeddingAdapter.cs:43-54): per component,
// |e| < ZeroThreshold (float compare) -> 0, else (long)(e * (double)GlobalScale). Entry for entry this
// is the dense form of EmbeddingAdapter.Quantize (:15-41) without a sparsity budget: Quantize drops
// exactly the components that are 0 here.
static void quantize_dense(const float* e, int64_t n, float zero_threshold, int64_t global_scale, int64_t* out) {
    const double scale = (double)global_scale;
    for (int64_t i = 0; i < n; i++) out[i] = std::fabs(e[i]) < zero_threshold ? 0 : cs_d2l((double)e[i] * scale);
}

// SparseVector.DistanceSquaredL2Fast (Math/SparseVector.cs:138-169) on dense vectors: the sparse
// merge adds (a-b)^2 where both are present and v^2 where one is, which is the dense sum over
// all dimensions; every square is (ulong)(diff * diff) with long wrap-around, summed in ulong.
static inline uint64_t distance_sq_l2_fast(const int64_t* a, const int64_t* b, int dim) {
    uint64_t sum = 0;
    for (int d = 0; d < dim; d++) {
        const int64_t diff = wrap_sub(a[d], b[d]);
        sum += (uint64_t)wrap_mul(diff, diff);
    }
    return sum;
}

// Exact k nearest database rows by DistanceSquaredL2Fast, ascending. RecallEvaluator.
// BruteForceKNearestL2 (Lattice/RecallEvaluator.cs:148-163) sorts all distances, and EmbeddingLattice.
// QueryKNearestL2 (Lattice/EmbeddingLattice.cs:70-77, KnnHeap :321-387) keeps the k smallest; both
// leave the order of equal distances to an unstable sort, so equal distances are ordered here by
// ascending row id. Rows past n (k > n) are reported as id -1, distance UINT64_MAX.
static void knn_l2(const int64_t* db, int64_t n, int dim, const int64_t* q, int nq, int k, int64_t id_base,
                   int64_t* ids, uint64_t* dist) {
#pragma omp parallel for schedule(dynamic, 1)
    for (int qi = 0; qi < nq; qi++) {
        std::vector<std::pair<uint64_t, int64_t>> best;  // max-heap of the k smallest (distance, id)
        best.reserve((size_t)k + 1);
        const int64_t* qv = q + (int64_t)qi * dim;
        for (int64_t r = 0; r < n; r++) {
            const std::pair<uint64_t, int64_t> e(distance_sq_l2_fast(qv, db + r * dim, dim), r + id_base);
            if ((int)best.size() < k) {
                best.push_back(e);
                std::push_heap(best.begin(), best.end());
            } else if (k > 0 && e < best.front()) {
                std::pop_heap(best.begin(), best.end());
                best.back() = e;
                std::push_heap(best.begin(), best.end());
            }
        }
        std::sort(best.begin(), best.end());
        for (int j = 0; j < k; j++) {
            const bool ok = j < (int)best.size();
            ids[(int64_t)qi * k + j] = ok ? best[j].second : -1;
            dist[(int64_t)qi * k + j] = ok ? best[j].first : UINT64_MAX;
        }
    }
}

// PredictNextToken with a VocabLattice (IntegerCausalSource.cs:149-157): the lattice holds the rows of
// TokenEmbeddingsFloat ((float)Half, :51-62) quantized by EmbeddingAdapter.Quantize with VocabLattice's
// options (ZeroThreshold 0.001, GlobalScale 1e9; Lattice/VocabLattice.cs:15-41); QueryTopK (:43-58)
// returns the k nearest by DistanceSquaredL2Fast; ScoreCandidates (:60-76) takes the sequential fp32
// dot of each candidate row with the hidden state and Array.Sort orders them by descending score.
// That sort is unstable, so equal scores have no defined order; here the first candidate (ascending
// distance, then id) among the highest scores wins. No candidate (k = 0) gives EOS.
static void vocab_lattice_build(const Causal& c);
static int32_t lattice_next(const Causal& c, const float* h, int k) {
    vocab_lattice_build(c);
    const int64_t V = (int64_t)c.vocab_q.size() / c.embd;
    std::vector<int64_t> hq(c.embd), ids(k > 0 ? k : 1);
    std::vector<uint64_t> dist(k > 0 ? k : 1);
    quantize_dense(h, c.embd, 0.001f, 1000000000LL, hq.data());
    if (k > 0) knn_l2(c.vocab_q.data(), V, c.embd, hq.data(), 1, k, 0, ids.data(), dist.data());
    int32_t best = c.eos;
    float best_score = 0.0f;
    bool have = false;
    for (int j = 0; j < k; j++) {
        if (ids[j] < 0) break;
        const uint16_t* row = c.tok.data() + ids[j] * c.embd;
        float dot = 0.0f;
        for (int d = 0; d < c.embd; d++) {
            float p = h[d] * half_to_float(row[d]);
            dot = dot + p;
        }
        if (!have || dot > best_score || (std::isnan(best_score) && !std::isnan(dot))) {
            best = (int32_t)ids[j];
            best_score = dot;
            have = true;
        }
    }
    return best;
}

static void vocab_lattice_build(const Causal& c) {
    if (!c.vocab_q.empty()) return;
    const int64_t rows = std::min<int64_t>(c.vocab, (int64_t)c.tok.size() / c.embd);
    std::vector<float> f((size_t)rows * c.embd);
    for (size_t i = 0; i < f.size(); i++) f[i] = half_to_float(c.tok[i]);
    c.vocab_q.resize(f.size());
    quantize_dense(f.data(), (int64_t)f.size(), 0.001f, 1000000000LL, c.vocab_q.data());
}

static int causal_next_lattice(const Causal& c, const int32_t* ids, int T, int k, int32_t* next) {
    std::vector<int64_t> x((size_t)T * c.embd);
    int st = causal_hidden(c, ids, T, -1, true, x.data());
    if (st) return st;
    const int64_t* last = x.data() + (size_t)(T - 1) * c.embd;
    std::vector<float> h(c.embd);
    double scale = std::pow(2.0, -c.scale_bits);
    for (int j = 0; j < c.embd; j++) h[j] = (float)((double)last[j] * scale);
    *next = lattice_next(c, h.data(), k);
    return SLXO_OK;
}

// ---------------------------------------------------------------------------------------------
// KD-tree lattice (EmbeddingLatticeBuilder, Lattice/EmbeddingLatticeBuilder.cs:11-127) and its
// SLAT wire format (SparseLatticeSerializer, Lattice/SparseLatticeSerializer.cs:5-166).
//
// The builder splits a span of occupants at the median of its highest-variance dimension:
// variance = sumSq * N - sum^2 over the span's N occupants (absent components are 0), among the
// dimensions some occupant of the span populates (:47-84); median = sorted values[N / 2] (:86-97);
// the span is partitioned in place by the two-pointer swap of :99-126 (values < median to the
// left); a span of at most LeafThreshold occupants, or one whose split leaves a side empty, or one
// with no populated dimension, becomes a leaf holding the span in its current order. The reference
// accumulates in BigInteger; here components are limited to |v| < 2^31 so Int128 is exact
// (N < 2^31). Equal variances: the reference takes the first in ConcurrentDictionary enumeration
// order (machine-dependent); here the lowest dimension.
struct TreeNode {
    int kind = 0;        // 0 leaf, 1 branch
    int mask = 0;        // branch: 1 below present, 2 above present
    int dim = 0;
    int64_t val = 0;
    int below = -1, above = -1;
    int64_t start = 0, count = 0;  // leaf: occupants perm[start .. start+count)
};
struct Tree {
    std::vector<TreeNode> nodes;
    std::vector<int64_t> perm;     // row ids in leaf order
    int root = -1;
};

static int tree_leaf(Tree& t, int64_t start, int64_t count) {
    TreeNode nd;
    nd.kind = 0;
    nd.start = start;
    nd.count = count;
    t.nodes.push_back(nd);
    return (int)t.nodes.size() - 1;
}

static int tree_build_rec(Tree& t, const int64_t* rows, int dim, int64_t start, int64_t len, int leaf_threshold) {
    int64_t* span = t.perm.data() + start;
    if (len <= leaf_threshold) return tree_leaf(t, start, len);
    int best_dim = -1;
    __int128 best_var = -1;
    for (int d = 0; d < dim; d++) {
        __int128 sum = 0, sq = 0;
        bool populated = false;
        for (int64_t i = 0; i < len; i++) {
            const int64_t v = rows[span[i] * dim + d];
            if (v != 0) populated = true;
            sum += v;
            sq += (__int128)v * v;
        }
        if (!populated) continue;
        const __int128 var = sq * len - sum * sum;
        if (var > best_var) {
            best_var = var;
            best_dim = d;
        }
    }
    if (best_dim < 0) return tree_leaf(t, start, len);
    std::vector<int64_t> vals((size_t)len);
    for (int64_t i = 0; i < len; i++) vals[i] = rows[span[i] * dim + best_dim];
    std::sort(vals.begin(), vals.end());
    const int64_t pivot = vals[(size_t)(len / 2)];
    int64_t left = 0, right = len - 1;
    while (left <= right) {
        if (rows[span[left] * dim + best_dim] < pivot) { left++; continue; }
        if (rows[span[right] * dim + best_dim] >= pivot) { right--; continue; }
        std::swap(span[left], span[right]);
        left++;
        right--;
    }
    const int64_t boundary = left;
    if (boundary == 0 || boundary == len) return tree_leaf(t, start, len);
    TreeNode br;
    br.kind = 1;
    br.mask = 3;
    br.dim = best_dim;
    br.val = pivot;
    t.nodes.push_back(br);
    const int id = (int)t.nodes.size() - 1;
    const int below = tree_build_rec(t, rows, dim, start, boundary, leaf_threshold);
    const int above = tree_build_rec(t, rows, dim, start + boundary, len - boundary, leaf_threshold);
    t.nodes[id].below = below;
    t.nodes[id].above = above;
    return id;
}

struct TreeStats { int64_t nodes = 0, branches = 0, leaves = 0, occupants = 0, max_depth = 0; };
static void tree_stats(const Tree& t, int node, int64_t depth, TreeStats& s) {
    const TreeNode& nd = t.nodes[node];
    s.nodes++;
    if (depth > s.max_depth) s.max_depth = depth;
    if (nd.kind == 0) {
        s.leaves++;
        s.occupants += nd.count;
        return;
    }
    s.branches++;
    if (nd.below >= 0) tree_stats(t, nd.below, depth + 1, s);
    if (nd.above >= 0) tree_stats(t, nd.above, depth + 1, s);
}

// Pre-order flattening (the order SparseLatticeSerializer.WriteNode visits, :64-95): per node its
// kind, child mask, split dimension and value, and for leaves the offset and count of its
// occupants in the leaf-order permutation.
static void tree_preorder(const Tree& t, int node, std::vector<int>& order) {
    order.push_back(node);
    const TreeNode& nd = t.nodes[node];
    if (nd.kind == 1) {
        if (nd.below >= 0) tree_preorder(t, nd.below, order);
        if (nd.above >= 0) tree_preorder(t, nd.above, order);
    }
}

struct ByteWriter {
    std::vector<uint8_t> b;
    template <class T> void put(T v) {
        const size_t o = b.size();
        b.resize(o + sizeof(T));
        memcpy(b.data() + o, &v, sizeof(T));
    }
};

// WriteNode / WriteLeaf (:64-114) with Int32PayloadSerializer (:187-194): occupant records carry
// TotalDimensions, the entry count and (ushort dimension, long value) for every nonzero component
// in ascending dimension (EmbeddingAdapter.Quantize keeps exactly the nonzero ones), then the payload.
static void slat_write_node(const Tree& t, int node, const int64_t* rows, int dim, const int32_t* payload,
                            ByteWriter& w) {
    const TreeNode& nd = t.nodes[node];
    if (nd.kind == 0) {
        w.put<uint8_t>(0);
        w.put<int32_t>((int32_t)nd.count);
        for (int64_t i = 0; i < nd.count; i++) {
            const int64_t r = t.perm[nd.start + i];
            const int64_t* v = rows + r * dim;
            int32_t nnz = 0;
            for (int d = 0; d < dim; d++) nnz += v[d] != 0;
            w.put<int32_t>(dim);
            w.put<int32_t>(nnz);
            for (int d = 0; d < dim; d++)
                if (v[d] != 0) {
                    w.put<uint16_t>((uint16_t)d);
                    w.put<int64_t>(v[d]);
                }
            w.put<int32_t>(payload[r]);
        }
        return;
    }
    w.put<uint8_t>(1);
    w.put<uint16_t>((uint16_t)nd.dim);
    w.put<int64_t>(nd.val);
    w.put<uint8_t>((uint8_t)nd.mask);
    if (nd.below >= 0) slat_write_node(t, nd.below, rows, dim, payload, w);
    if (nd.above >= 0) slat_write_node(t, nd.above, rows, dim, payload, w);
}

// Load (:46-62, ReadNode/ReadLeaf/ReadBranch :116-166): magic and version checks
// (InvalidDataException), unknown tags (InvalidDataException), short input (EndOfStreamException),
// and the SparseVector constructor's checks on every occupant (Math/SparseVector.cs:21-28,303-320:
// TotalDimensions > 0, dimensions below it, ascending without duplicates, no zero values:
// ArgumentException). Occupants become dense rows of width `dim` (all occupants must share it).
struct SlatReader {
    const uint8_t* p;
    int64_t n, pos = 0;
    int status = SLXO_OK;
    template <class T> bool get(T& v) {
        if (status) return false;
        if (pos + (int64_t)sizeof(T) > n) { status = SLXO_EEOF; return false; }
        memcpy(&v, p + pos, sizeof(T));
        pos += sizeof(T);
        return true;
    }
};
struct SlatLoaded {
    Tree t;
    std::vector<int64_t> rows;    // [n][dim]
    std::vector<int32_t> payload; // [n]
    int dim = -1;
};
static int slat_read_node(SlatReader& r, SlatLoaded& out) {
    uint8_t tag;
    if (!r.get(tag)) return -1;
    if (tag == 0) {
        int32_t count;
        if (!r.get(count)) return -1;
        if (count < 0) { r.status = SLXO_EFORMAT; return -1; }
        const int64_t start = (int64_t)out.t.perm.size();
        for (int32_t i = 0; i < count; i++) {
            int32_t total, entries;
            if (!r.get(total) || !r.get(entries)) return -1;
            if (total <= 0 || entries < 0) { r.status = SLXO_EINVAL; return -1; }
            if (out.dim < 0) out.dim = total;
            if (total != out.dim) { r.status = SLXO_EINVAL; return -1; }
            const int64_t row = (int64_t)out.payload.size();
            out.rows.resize((size_t)(row + 1) * total, 0);
            int prev = -1;
            for (int32_t e = 0; e < entries; e++) {
                uint16_t d;
                int64_t v;
                if (!r.get(d) || !r.get(v)) return -1;
                if ((int)d >= total || v == 0 || (int)d <= prev) { r.status = SLXO_EINVAL; return -1; }
                prev = d;
                out.rows[(size_t)row * total + d] = v;
            }
            int32_t pay;
            if (!r.get(pay)) return -1;
            out.payload.push_back(pay);
            out.t.perm.push_back(row);
        }
        return tree_leaf(out.t, start, count);
    }
    if (tag == 1) {
        uint16_t d;
        int64_t v;
        uint8_t mask;
        if (!r.get(d) || !r.get(v) || !r.get(mask)) return -1;
        TreeNode br;
        br.kind = 1;
        br.dim = d;
        br.val = v;
        br.mask = mask & 3;
        out.t.nodes.push_back(br);
        const int id = (int)out.t.nodes.size() - 1;
        int below = -1, above = -1;
        if (mask & 1) { below = slat_read_node(r, out); if (below < 0) return -1; }
        if (mask & 2) { above = slat_read_node(r, out); if (above < 0) return -1; }
        out.t.nodes[id].below = below;
        out.t.nodes[id].above = above;
        return id;
    }
    r.status = SLXO_EFORMAT;
    return -1;
}

static void tree_export(const Tree& t, int32_t* kind, int32_t* mask, int32_t* dim, int64_t* val, int64_t* start,
                        int64_t* count) {
    std::vector<int> order;
    if (t.root >= 0) tree_preorder(t, t.root, order);
    for (size_t i = 0; i < order.size(); i++) {
        const TreeNode& nd = t.nodes[order[i]];
        kind[i] = nd.kind;
        mask[i] = nd.mask;
        dim[i] = nd.dim;
        val[i] = nd.val;
        start[i] = nd.start;
        count[i] = nd.count;
    }
}

// ---------------------------------------------------------------------------------------------
// TransformerEmbeddingSource: the float twin of the encoder (Gguf/TransformerEmbeddingSource.cs).
// Weights are the GGUF tensors read as float (ReadTensorF32, :514-557); the forward (:124-141)
// runs BuildEmbeddings (:144-163), LayerNorm with eps 1e-12 (:380-408; the GGUF epsilon is read
// but unused), the blocks (:166-211: QKV, float RoPE from a 512-row cache :227-275, attention
// :337-378 with MathF.Exp softmax :440-460, O, residual, LayerNorm, SiLU-gated FFN :461, residual,
// LayerNorm), MeanPool over all rows (:474-491) and L2Normalize (:493-503). The reference's dots
// are Vector<float> SIMD (lane order machine-dependent); here they are sequential fp32 with separate
// multiply and add, so the restatement agrees with the reference to rounding, not bit for bit.
struct FloatLayer { std::vector<float> qkv, o, anw, anb, up, gate, down, lnw, lnb; };
struct FloatEncoder {
    int embd = 0, heads = 0, layers = 0, ff = 0, unk = 0;
    std::vector<float> tok, tt, enw, enb, cs, sn;
    std::vector<FloatLayer> L;
};

static FloatEncoder* float_encoder_load(const char* path, int* status) {
    std::unique_ptr<Gguf> g(gguf_open(path, status));
    if (!g) return nullptr;
    std::string al = g->arch;
    std::transform(al.begin(), al.end(), al.begin(), ::tolower);
    if (al != "nomic-bert" && al != "bert") { *status = SLXO_EUNSUPPORTED; return nullptr; }
    std::unique_ptr<FloatEncoder> e(new FloatEncoder());
    e->embd = g->embd; e->heads = g->heads; e->layers = g->layers; e->ff = g->ff;
    const float base = meta_float(*g, g->arch + ".rope.freq_base", 10000.0f);
    int st;
    if ((st = gguf_read_f32(g.get(), "token_embd.weight", e->tok))) { *status = st; return nullptr; }
    std::vector<float> tt;
    if ((st = gguf_read_f32(g.get(), "token_types.weight", tt))) { *status = st; return nullptr; }
    if ((int64_t)tt.size() < e->embd) { *status = SLXO_EINVAL; return nullptr; }
    e->tt.assign(tt.begin(), tt.begin() + e->embd);
    if ((st = gguf_read_f32(g.get(), "token_embd_norm.weight", e->enw))) { *status = st; return nullptr; }
    if ((st = gguf_read_f32(g.get(), "token_embd_norm.bias", e->enb))) { *status = st; return nullptr; }
    e->L.resize(e->layers);
    for (int i = 0; i < e->layers; i++) {
        std::string p = "blk." + std::to_string(i);
        FloatLayer& l = e->L[i];
        const char* names[9] = {".attn_qkv.weight", ".attn_output.weight", ".attn_output_norm.weight",
                                ".attn_output_norm.bias", ".ffn_up.weight", ".ffn_gate.weight", ".ffn_down.weight",
                                ".layer_output_norm.weight", ".layer_output_norm.bias"};
        std::vector<float>* dst[9] = {&l.qkv, &l.o, &l.anw, &l.anb, &l.up, &l.gate, &l.down, &l.lnw, &l.lnb};
        for (int j = 0; j < 9; j++)
            if ((st = gguf_read_f32(g.get(), p + names[j], *dst[j]))) { *status = st; return nullptr; }
    }
    if (g->n_tokens == 0) { *status = SLXO_EINVAL; return nullptr; }
    e->unk = g->unk;
    // RopeCache (:227-252): theta = (float)Pow(base, -2i/hd), angle = t * theta in double.
    const int hd = e->embd / e->heads, half = hd / 2;
    e->cs.resize((size_t)512 * half);
    e->sn.resize((size_t)512 * half);
    for (int t = 0; t < 512; t++)
        for (int i = 0; i < half; i++) {
            const float theta = (float)std::pow((double)base, -2.0 * i / hd);
            const double angle = t * (double)theta;
            e->cs[(size_t)t * half + i] = (float)std::cos(angle);
            e->sn[(size_t)t * half + i] = (float)std::sin(angle);
        }
    *status = SLXO_OK;
    return e.release();
}

static float fdot(const float* a, const float* b, int n) {
    float s = 0.0f;
    for (int i = 0; i < n; i++) s = s + a[i] * b[i];
    return s;
}

static void f_matmul(const float* a, int rows, int nin, const float* w, int nout, float* c) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++)
        for (int o = 0; o < nout; o++) c[(size_t)r * nout + o] = fdot(a + (size_t)r * nin, w + (size_t)o * nin, nin);
}

static void f_layernorm(float* x, int T, int d, const float* w, const float* b) {
    for (int t = 0; t < T; t++) {
        float* r = x + (size_t)t * d;
        float mean = 0.0f;
        for (int j = 0; j < d; j++) mean += r[j];
        mean /= d;
        float var = 0.0f;
        for (int j = 0; j < d; j++) {
            const float dl = r[j] - mean;
            var += dl * dl;
        }
        var /= d;
        const float inv = 1.0f / std::sqrt(var + 1e-12f);
        for (int j = 0; j < d; j++) r[j] = (r[j] - mean) * inv * w[j] + b[j];
    }
}

static int float_encoder_forward(const FloatEncoder& e, const int32_t* ids, int T, float* out) {
    const int d = e.embd, H = e.heads, hd = d / H, half = hd / 2, F = e.ff;
    if (T > 512) return SLXO_ERANGE;  // the 512-row RoPE cache
    std::vector<float> x((size_t)T * d);
    for (int t = 0; t < T; t++) {
        int64_t src = (int64_t)ids[t] * d;
        if (ids[t] < 0 || src + d > (int64_t)e.tok.size()) src = (int64_t)e.unk * d;
        for (int j = 0; j < d; j++) x[(size_t)t * d + j] = e.tok[src + j] + e.tt[j];
    }
    f_layernorm(x.data(), T, d, e.enw.data(), e.enb.data());
    std::vector<float> qkv((size_t)T * 3 * d), q((size_t)T * d), k((size_t)T * d), v((size_t)T * d), att((size_t)T * d),
        proj((size_t)T * d), up((size_t)T * F), gate((size_t)T * F), down((size_t)T * d), sc((size_t)T * T);
    for (int l = 0; l < e.layers; l++) {
        const FloatLayer& L = e.L[l];
        f_matmul(x.data(), T, d, L.qkv.data(), 3 * d, qkv.data());
        for (int t = 0; t < T; t++)
            for (int j = 0; j < d; j++) {
                q[(size_t)t * d + j] = qkv[(size_t)t * 3 * d + j];
                k[(size_t)t * d + j] = qkv[(size_t)t * 3 * d + d + j];
                v[(size_t)t * d + j] = qkv[(size_t)t * 3 * d + 2 * d + j];
            }
        for (float* m : {q.data(), k.data()})
            for (int t = 0; t < T; t++)
                for (int h = 0; h < H; h++)
                    for (int i = 0; i < half; i++) {
                        const float c = e.cs[(size_t)t * half + i], s_ = e.sn[(size_t)t * half + i];
                        float* p = m + (size_t)t * d + h * hd;
                        const float x0 = p[i], x1 = p[i + half];
                        p[i] = x0 * c - x1 * s_;
                        p[i + half] = x0 * s_ + x1 * c;
                    }
        const float scale = 1.0f / std::sqrt((float)hd);
        std::fill(att.begin(), att.end(), 0.0f);
        for (int h = 0; h < H; h++) {
            for (int t = 0; t < T; t++)
                for (int s2 = 0; s2 < T; s2++)
                    sc[(size_t)t * T + s2] = fdot(&q[(size_t)t * d + h * hd], &k[(size_t)s2 * d + h * hd], hd) * scale;
            for (int t = 0; t < T; t++) {
                float* r = &sc[(size_t)t * T];
                float mx = r[0];
                for (int s2 = 1; s2 < T; s2++) mx = r[s2] > mx ? r[s2] : mx;
                float sum = 0.0f;
                for (int s2 = 0; s2 < T; s2++) {
                    r[s2] = std::exp(r[s2] - mx);
                    sum += r[s2];
                }
                const float inv = 1.0f / sum;
                for (int s2 = 0; s2 < T; s2++) r[s2] *= inv;
            }
            for (int t = 0; t < T; t++)
                for (int s2 = 0; s2 < T; s2++) {
                    const float w = sc[(size_t)t * T + s2];
                    for (int j = 0; j < hd; j++) att[(size_t)t * d + h * hd + j] += w * v[(size_t)s2 * d + h * hd + j];
                }
        }
        f_matmul(att.data(), T, d, L.o.data(), d, proj.data());
        for (size_t i = 0; i < proj.size(); i++) proj[i] += x[i];
        f_layernorm(proj.data(), T, d, L.anw.data(), L.anb.data());
        f_matmul(proj.data(), T, d, L.up.data(), F, up.data());
        f_matmul(proj.data(), T, d, L.gate.data(), F, gate.data());
        for (size_t i = 0; i < up.size(); i++) up[i] *= gate[i] / (1.0f + std::exp(-gate[i]));
        f_matmul(up.data(), T, F, L.down.data(), d, down.data());
        for (size_t i = 0; i < down.size(); i++) down[i] += proj[i];
        f_layernorm(down.data(), T, d, L.lnw.data(), L.lnb.data());
        x.swap(down);
    }
    std::vector<float> pooled((size_t)d, 0.0f);
    for (int t = 0; t < T; t++)
        for (int j = 0; j < d; j++) pooled[j] += x[(size_t)t * d + j];
    const float inv = 1.0f / T;
    for (int j = 0; j < d; j++) pooled[j] *= inv;
    float norm = 0.0f;
    for (int j = 0; j < d; j++) norm += pooled[j] * pooled[j];
    norm = std::sqrt(norm);
    if (norm >= 1e-10f) {
        const float in = 1.0f / norm;
        for (int j = 0; j < d; j++) pooled[j] *= in;
    }
    memcpy(out, pooled.data(), sizeof(float) * d);
    return SLXO_OK;
}

extern "C" {

int slxo_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}

float slxo_half_to_float(uint16_t h) { return half_to_float(h); }
uint16_t slxo_float_to_half(float f) { return float_to_half(f); }
void slxo_half_to_float_n(const uint16_t* h, int64_t n, float* out) { for (int64_t i = 0; i < n; i++) out[i] = half_to_float(h[i]); }
void slxo_float_to_half_n(const float* f, int64_t n, uint16_t* out) { for (int64_t i = 0; i < n; i++) out[i] = float_to_half(f[i]); }

int slxo_dequantize(int dtype, const uint8_t* raw, int64_t len, float* out, int64_t n) {
    return dequantize((uint32_t)dtype, raw, len, out, n);
}
int64_t slxo_byte_count(int dtype, int64_t elements) { return gguf_byte_count((uint32_t)dtype, elements); }

void slxo_quantize_from_float(const float* src, int64_t n, int bits, int64_t* out) { quantize_from_float(src, n, bits, out); }

void slxo_dot_int128(const int64_t* a, const int64_t* b, int n, int64_t* lo_hi) {
    i128 r = dot_i128(a, b, n);
    lo_hi[0] = lo64(r);
    lo_hi[1] = lo64(r >> 64);
}
void slxo_matmul_long(const int64_t* a, int rows, int cols, const int64_t* w, int colsB, int shift, int64_t* c) {
    matmul_long(a, rows, cols, w, colsB, shift, c);
}
void slxo_matmul_half(const int64_t* a, int rows, int cols, const uint16_t* w, int colsB, int scale_bits, int shift, int64_t* c) {
    matmul_half(a, rows, cols, w, colsB, scale_bits, shift, c);
}
void slxo_matmul_float(const int64_t* a, int rows, int cols, const float* w, int colsB, int scale_bits, int shift, int64_t* c) {
    matmul_float(a, rows, cols, w, colsB, scale_bits, shift, c);
}

int64_t slxo_fixed_exp(int64_t x, int frac) { return fixed_exp(x, frac); }
int64_t slxo_fixed_sigmoid(int64_t x, int frac) { return fixed_sigmoid(x, frac); }
int64_t slxo_fixed_silu(int64_t x, int frac) { return fixed_silu(x, frac); }
void slxo_fixed_softmax(int64_t* s, int len, int frac) { fixed_softmax(s, len, frac); }
int64_t slxo_isqrt64(int64_t v) { return isqrt64(v); }
int64_t slxo_isqrt128(int64_t lo, int64_t hi) { return isqrt128((i128)(((u128)(uint64_t)hi << 64) | (uint64_t)lo)); }

void slxo_layernorm(int64_t* x, int seq, int embd, const int64_t* w, const int64_t* b) { layernorm(x, seq, embd, w, b); }
void slxo_rmsnorm(int64_t* x, int seq, int embd, const int64_t* w) { rmsnorm(x, seq, embd, w); }
void slxo_rmsnorm_per_head(int64_t* x, int seq, int nh, int hd, const int64_t* w) { rmsnorm_per_head(x, seq, nh, hd, w); }

void slxo_rope_cache(int max_seq, int head_dim, float base, int frac, int64_t* cos_out, int64_t* sin_out) {
    RoPE c;
    rope_build(c, max_seq, head_dim, base, frac);
    memcpy(cos_out, c.cos.data(), sizeof(int64_t) * c.cos.size());
    memcpy(sin_out, c.sin.data(), sizeof(int64_t) * c.sin.size());
}
int slxo_apply_rope(int64_t* x, int seq, int embd, int nh, int max_seq, int head_dim, float base, int frac) {
    RoPE c;
    rope_build(c, max_seq, head_dim, base, frac);
    return apply_rope(x, seq, embd, nh, c);
}
void slxo_attention(const int64_t* q, const int64_t* k, const int64_t* v, int seq, int q_embd, int kv_dim, int nh,
                    int nkv, int scale_exp, int frac, int mode, int window, int64_t* out) {
    gqa(q, k, v, seq, q_embd, kv_dim, nh, nkv, scale_exp, frac, mode, window, out);
}
void slxo_silu_gate(const int64_t* gate, int64_t* up, int64_t n, int frac) { silu_gate(gate, up, n, frac); }
void slxo_ffn_long(const int64_t* x, int seq, int embd, const int64_t* wg, const int64_t* wu, const int64_t* wd, int nff,
                   int shift, int frac, int64_t* out) {
    ffn_long(x, seq, embd, wg, wu, wd, nff, shift, frac, out);
}
void slxo_ffn_half(const int64_t* x, int seq, int embd, const uint16_t* wg, const uint16_t* wu, const uint16_t* wd,
                   int nff, int scale_bits, int frac, int64_t* out) {
    ffn_half(x, seq, embd, wg, wu, wd, nff, scale_bits, frac, out);
}
void slxo_mean_pool(const int64_t* x, int T, int d, int64_t* pooled) { mean_pool(x, T, d, pooled); }
void slxo_to_float_l2(const int64_t* v, int d, int scale_bits, float* out) { to_float_l2(v, d, scale_bits, out); }
int slxo_argmax_half(const float* h, const uint16_t* E, int64_t n_elems, int vocab, int dims) {
    return argmax_half(h, E, n_elems, vocab, dims);
}

// ---- GGUF ----
void* slxo_gguf_open(const char* path, int* status) { return gguf_open(path, status); }
void slxo_gguf_close(void* g) { delete (Gguf*)g; }
int slxo_gguf_info(void* gp, int* out) {  // version, embd, ctx, heads, layers, ff, n_tokens, bos, eos, unk, n_tensors
    Gguf* g = (Gguf*)gp;
    int v[11] = {(int)g->version, g->embd, g->ctx, g->heads, g->layers, g->ff, g->n_tokens, g->bos, g->eos, g->unk,
                 (int)g->tensors.size()};
    memcpy(out, v, sizeof(v));
    return SLXO_OK;
}
int64_t slxo_gguf_data_offset(void* g) { return ((Gguf*)g)->data_offset; }
int slxo_gguf_arch(void* g, char* buf, int cap) {
    const std::string& a = ((Gguf*)g)->arch;
    snprintf(buf, (size_t)cap, "%s", a.c_str());
    return (int)a.size();
}
int64_t slxo_gguf_tensor_elements(void* gp, const char* name) {
    Gguf* g = (Gguf*)gp;
    auto it = g->index.find(name);
    return it == g->index.end() ? -1 : g->tensors[it->second].elements;
}
int slxo_gguf_tensor_dtype(void* gp, const char* name) {
    Gguf* g = (Gguf*)gp;
    auto it = g->index.find(name);
    return it == g->index.end() ? -1 : (int)g->tensors[it->second].dtype;
}
int slxo_gguf_read_f32(void* gp, const char* name, float* out, int64_t cap) {
    std::vector<float> f;
    int st = gguf_read_f32((Gguf*)gp, name, f);
    if (st) return st;
    if ((int64_t)f.size() > cap) return SLXO_EINVAL;
    memcpy(out, f.data(), sizeof(float) * f.size());
    return SLXO_OK;
}

// ---- encoder ----
void* slxo_encoder_load(const char* path, int scale_bits, int* status) { return encoder_load(path, scale_bits, status); }
void slxo_encoder_free(void* e) { delete (Encoder*)e; }
int slxo_encoder_info(void* ep, int* out) {
    Encoder* e = (Encoder*)ep;
    out[0] = e->embd; out[1] = e->heads; out[2] = e->layers; out[3] = e->ff; out[4] = e->unk;
    out[5] = (int)(e->vocab_rows / std::max(1, e->embd));
    return SLXO_OK;
}
int slxo_encoder_hidden(void* ep, const int32_t* ids, int T, int n_layers, int64_t* x) {
    Encoder* e = (Encoder*)ep;
    return encoder_hidden(*e, ids, T, n_layers, x);
}
// Forward (IntegerTransformerSource.cs:65-78) for B independent sequences of T tokens (the
// reference's EmbedBatchAsync is a sequential loop over texts, IntegerTransformerSource.cs:40-47).
int slxo_encoder_forward(void* ep, const int32_t* ids, int B, int T, int64_t* pooled) {
    Encoder* e = (Encoder*)ep;
    std::vector<int64_t> x((size_t)T * e->embd);
    for (int b = 0; b < B; b++) {
        int st = encoder_hidden(*e, ids + (int64_t)b * T, T, -1, x.data());
        if (st) return st;
        mean_pool(x.data(), T, e->embd, pooled + (int64_t)b * e->embd);
    }
    return SLXO_OK;
}

// ---- causal LM ----
void* slxo_causal_load(const char* path, int scale_bits, int* status) { return causal_load(path, scale_bits, status, false); }
void* slxo_gemma_encoder_load(const char* path, int scale_bits, int* status) {
    return causal_load(path, scale_bits, status, true);
}
void slxo_causal_free(void* c) { delete (Causal*)c; }
int slxo_causal_info(void* cp, int* out) {
    Causal* c = (Causal*)cp;
    int v[12] = {c->embd, c->heads, c->kv_heads, c->head_dim, c->ff, c->layers, c->vocab, c->sliding, c->eos, c->unk,
                 c->q_dim, c->kv_dim};
    memcpy(out, v, sizeof(v));
    return SLXO_OK;
}
int slxo_causal_hidden(void* cp, const int32_t* ids, int T, int n_layers, int final_norm, int64_t* x) {
    return causal_hidden(*(Causal*)cp, ids, T, n_layers, final_norm != 0, x);
}
int slxo_causal_forward_last(void* cp, const int32_t* ids, int T, int64_t* last) {
    Causal* c = (Causal*)cp;
    std::vector<int64_t> x((size_t)T * c->embd);
    int st = causal_hidden(*c, ids, T, -1, true, x.data());
    if (st) return st;
    memcpy(last, x.data() + (size_t)(T - 1) * c->embd, sizeof(int64_t) * c->embd);
    return SLXO_OK;
}
int slxo_causal_next_token(void* cp, const int32_t* ids, int T, int32_t* next) {
    return causal_next(*(Causal*)cp, ids, T, next, nullptr);
}
int slxo_causal_next_token_lattice(void* cp, const int32_t* ids, int T, int k, int32_t* next) {
    return causal_next_lattice(*(Causal*)cp, ids, T, k, next);
}
// Generate(useLattice: true, latticeK: k) on token ids (IntegerCausalSource.cs:86-108).
int slxo_causal_generate_lattice(void* cp, const int32_t* ids, int T, int max_new, int k, int32_t* out, int* n_out) {
    Causal* c = (Causal*)cp;
    std::vector<int32_t> seq(ids, ids + T);
    *n_out = 0;
    for (int step = 0; step < max_new; step++) {
        int32_t nx;
        int st = causal_next_lattice(*c, seq.data(), (int)seq.size(), k, &nx);
        if (st) return st;
        if (nx == c->eos) break;
        seq.push_back(nx);
        out[(*n_out)++] = nx;
    }
    return SLXO_OK;
}
// Generate (IntegerCausalSource.cs:86-108) on token ids: full re-forward per step, greedy argmax,
// stop at EOS (not appended). Returns the new ids in out[0..*n_out).
int slxo_causal_generate(void* cp, const int32_t* ids, int T, int max_new, int32_t* out, int* n_out) {
    Causal* c = (Causal*)cp;
    std::vector<int32_t> seq(ids, ids + T);
    *n_out = 0;
    for (int step = 0; step < max_new; step++) {
        int32_t nx;
        int st = causal_next(*c, seq.data(), (int)seq.size(), &nx, nullptr);
        if (st) return st;
        if (nx == c->eos) break;
        seq.push_back(nx);
        out[(*n_out)++] = nx;
    }
    return SLXO_OK;
}
// IntegerGemmaSource.Forward (IntegerGemmaSource.cs:66-80): non-causal, output norm, mean pool.
int slxo_gemma_encoder_forward(void* cp, const int32_t* ids, int B, int T, int64_t* pooled) {
    Causal* c = (Causal*)cp;
    std::vector<int64_t> x((size_t)T * c->embd);
    for (int b = 0; b < B; b++) {
        int st = causal_hidden(*c, ids + (int64_t)b * T, T, -1, true, x.data());
        if (st) return st;
        mean_pool(x.data(), T, c->embd, pooled + (int64_t)b * c->embd);
    }
    return SLXO_OK;
}

// ---- lattice k-NN ----
void slxo_quantize_dense(const float* e, int64_t n, float zero_threshold, int64_t global_scale, int64_t* out) {
    quantize_dense(e, n, zero_threshold, global_scale, out);
}
uint64_t slxo_distance_sq_l2_fast(const int64_t* a, const int64_t* b, int dim) { return distance_sq_l2_fast(a, b, dim); }
void slxo_knn_l2(const int64_t* db, int64_t n, int dim, const int64_t* q, int nq, int k, int64_t id_base, int64_t* ids,
                 uint64_t* dist) {
    knn_l2(db, n, dim, q, nq, k, id_base, ids, dist);
}


// ---- KD-tree lattice and SLAT (test oracle) -------------------------------------------------
void* slxo_tree_build(const int64_t* rows, int64_t n, int dim, int leaf_threshold, int* status) {
    *status = SLXO_OK;
    if (n < 0 || dim <= 0 || dim > 65536 || (n > 0 && !rows)) { *status = SLXO_EINVAL; return nullptr; }
    for (int64_t i = 0; i < n * dim; i++)
        if (rows[i] <= -(1LL << 31) || rows[i] >= (1LL << 31)) { *status = SLXO_ERANGE; return nullptr; }
    Tree* t = new Tree();
    t->perm.resize((size_t)n);
    for (int64_t i = 0; i < n; i++) t->perm[i] = i;
    t->root = tree_build_rec(*t, rows, dim, 0, n, leaf_threshold);
    return t;
}
void slxo_tree_free(void* h) { delete (Tree*)h; }
// info: nodes, branches, leaves, occupants, max depth
void slxo_tree_info(void* h, int64_t* info) {
    TreeStats s;
    Tree* t = (Tree*)h;
    if (t->root >= 0) tree_stats(*t, t->root, 0, s);
    info[0] = s.nodes; info[1] = s.branches; info[2] = s.leaves; info[3] = s.occupants; info[4] = s.max_depth;
}
void slxo_tree_export(void* h, int32_t* kind, int32_t* mask, int32_t* dim, int64_t* val, int64_t* start,
                      int64_t* count, int64_t* perm) {
    Tree* t = (Tree*)h;
    tree_export(*t, kind, mask, dim, val, start, count);
    for (size_t i = 0; i < t->perm.size(); i++) perm[i] = t->perm[i];
}
// SLAT bytes of a built tree over `rows` with Int32 payloads; returns the size (call with
// out = nullptr to size the buffer).
int64_t slxo_slat_save(void* h, const int64_t* rows, int dim, const int32_t* payload, uint8_t* out, int64_t cap) {
    Tree* t = (Tree*)h;
    ByteWriter w;
    w.put<uint32_t>(0x544C4153u);
    w.put<uint16_t>(1);
    if (t->root >= 0) slat_write_node(*t, t->root, rows, dim, payload, w);
    if (out && cap >= (int64_t)w.b.size()) memcpy(out, w.b.data(), w.b.size());
    return (int64_t)w.b.size();
}
// Parses SLAT bytes; on success *n_out rows of *dim_out components (dim 0 when the file holds no
// occupant) are available through slxo_slat_rows and the tree through slxo_tree_*.
void* slxo_slat_load(const uint8_t* bytes, int64_t n, int* status, int64_t* n_out, int* dim_out) {
    SlatReader r{bytes, n};
    uint32_t magic;
    uint16_t version;
    *status = SLXO_OK;
    if (!r.get(magic)) { *status = r.status; return nullptr; }
    if (magic != 0x544C4153u) { *status = SLXO_EFORMAT; return nullptr; }
    if (!r.get(version)) { *status = r.status; return nullptr; }
    if (version != 1) { *status = SLXO_EFORMAT; return nullptr; }
    SlatLoaded* L = new SlatLoaded();
    L->t.root = slat_read_node(r, *L);
    if (L->t.root < 0) {
        *status = r.status ? r.status : SLXO_EFORMAT;
        delete L;
        return nullptr;
    }
    *n_out = (int64_t)L->payload.size();
    *dim_out = L->dim < 0 ? 0 : L->dim;
    return L;
}
void* slxo_slat_tree(void* h) { return &((SlatLoaded*)h)->t; }
void slxo_slat_rows(void* h, int64_t* rows, int32_t* payload) {
    SlatLoaded* L = (SlatLoaded*)h;
    memcpy(rows, L->rows.data(), L->rows.size() * sizeof(int64_t));
    memcpy(payload, L->payload.data(), L->payload.size() * sizeof(int32_t));
}
void slxo_slat_free(void* h) { delete (SlatLoaded*)h; }

// ---- float encoder twin (test oracle) ---------------------------------------------------------
void* slxo_float_encoder_load(const char* path, int* status) { return float_encoder_load(path, status); }
void slxo_float_encoder_free(void* h) { delete (FloatEncoder*)h; }
int slxo_float_encoder_forward(void* h, const int32_t* ids, int T, float* out) {
    return float_encoder_forward(*(FloatEncoder*)h, ids, T, out);
}
}  // extern "C"
