// gguf.cpp -- GGUF container parsing for libslx (see gguf.hpp for the reference it follows).
#include "gguf.hpp"

#include <cstring>

#include "slx_status.h"

namespace slx {

int64_t gguf_byte_count(uint32_t dtype, int64_t e) {
    switch (dtype) {
        case GG_F32: return e * 4;
        case GG_F16: case GG_BF16: return e * 2;
        case GG_Q8_0: return (e / 32) * 34;
        case GG_Q4_0: return (e / 32) * 18;
        case GG_Q4_1: return (e / 32) * 20;
        case GG_Q5_0: return (e / 32) * 22;
        case GG_Q5_1: return (e / 32) * 24;
        case GG_Q2_K: return (e / 256) * 84;
        case GG_Q3_K: return (e / 256) * 110;
        case GG_Q4_K: return (e / 256) * 144;
        case GG_Q5_K: return (e / 256) * 176;
        case GG_Q6_K: return (e / 256) * 210;
        case GG_Q8_K: return (e / 256) * 292;
        case GG_MXFP4: return (e / 32) * 17;
        default: return e * 4;
    }
}

int64_t gguf_decode_bytes(uint32_t dtype, int64_t e) {
    switch (dtype) {
        case GG_F32: case GG_F16: case GG_BF16: case GG_Q8_0: case GG_Q4_0: case GG_MXFP4:
        case GG_Q2_K: case GG_Q3_K: case GG_Q4_K: case GG_Q5_K: case GG_Q6_K: case GG_Q8_K:
            return gguf_byte_count(dtype, e);
        default: return -1;  // Q4_1/Q5_0/Q5_1 are sized but not decodable (GgufReader.cs:195-197)
    }
}

namespace {
struct Reader {
    FILE* fp;
    bool eof = false;
    void raw(void* p, size_t n) {
        if (!eof && fread(p, 1, n, fp) != n) eof = true;
        if (eof) memset(p, 0, n);
    }
    uint8_t u8() { uint8_t v; raw(&v, 1); return v; }
    uint16_t u16() { uint16_t v; raw(&v, 2); return v; }
    uint32_t u32() { uint32_t v; raw(&v, 4); return v; }
    uint64_t u64() { uint64_t v; raw(&v, 8); return v; }
    bool str(std::string& s) {
        uint64_t n = u64();
        s.clear();
        if (eof || n == 0) return !eof;
        if (n > (1ull << 31)) { eof = true; return false; }
        s.resize(n);
        raw(&s[0], n);
        return !eof;
    }
};

// Reads one value; arrays keep only their length and element type (strings are skipped), except
// that the caller can ask for the element count. Returns false on an unknown type id.
bool read_value(Reader& r, uint32_t t, GgufValue& v) {
    v.type = t;
    switch (t) {
        case 0: v.u = r.u8(); v.i = (int64_t)v.u; return true;
        case 1: v.i = (int8_t)r.u8(); v.u = (uint64_t)v.i; return true;
        case 2: v.u = r.u16(); v.i = (int64_t)v.u; return true;
        case 3: v.i = (int16_t)r.u16(); v.u = (uint64_t)v.i; return true;
        case 4: v.u = r.u32(); v.i = (int64_t)v.u; return true;
        case 5: v.i = (int32_t)r.u32(); v.u = (uint64_t)v.i; return true;
        case 6: { uint32_t b = r.u32(); float f; memcpy(&f, &b, 4); v.f = f; return true; }
        case 7: v.u = r.u8() != 0; v.i = (int64_t)v.u; return true;
        case 8: r.str(v.s); return true;
        case 9: {
            v.array_type = r.u32();
            v.array_len = r.u64();
            if (r.eof) return true;
            GgufValue item;
            for (uint64_t k = 0; k < v.array_len && !r.eof; k++)
                if (!read_value(r, v.array_type, item)) return false;
            return true;
        }
        case 10: v.u = r.u64(); v.i = (int64_t)v.u; return true;
        case 11: v.i = (int64_t)r.u64(); v.u = (uint64_t)v.i; return true;
        case 12: { uint64_t b = r.u64(); memcpy(&v.f, &b, 8); return true; }
        default: return false;
    }
}
}  // namespace

GgufFile::~GgufFile() {
    if (fp_) fclose(fp_);
}

int GgufFile::open(const std::string& path, std::string& err) {
    fp_ = fopen(path.c_str(), "rb");
    if (!fp_) { err = "GGUF file not found: " + path; return SLX_ENOTFOUND; }
    Reader r{fp_};
    uint32_t magic = r.u32();
    if (r.eof) { err = "unexpected end of GGUF header"; return SLX_EEOF; }
    if (magic != 0x46554747u) { err = "Not a GGUF file: bad magic"; return SLX_EFORMAT; }
    version = r.u32();
    if (r.eof) { err = "unexpected end of GGUF header"; return SLX_EEOF; }
    if (version != 2 && version != 3) { err = "Unsupported GGUF version " + std::to_string(version); return SLX_EFORMAT; }
    uint64_t n_tensors = r.u64(), n_meta = r.u64();
    for (uint64_t i = 0; i < n_meta && !r.eof; i++) {
        std::string key;
        r.str(key);
        uint32_t t = r.u32();
        GgufValue v;
        if (!read_value(r, t, v)) { err = "Unknown GGUF value type " + std::to_string(t); return SLX_EFORMAT; }
        meta[key] = v;
    }
    for (uint64_t i = 0; i < n_tensors && !r.eof; i++) {
        GgufTensor t;
        r.str(t.name);
        uint32_t nd = r.u32();
        if (nd > 64) { err = "bad tensor rank"; return SLX_EFORMAT; }
        t.shape.resize(nd);
        int64_t e = 1;
        for (uint32_t d = 0; d < nd; d++) { t.shape[d] = (int)r.u64(); e *= t.shape[d]; }
        t.dtype = r.u32();
        t.offset = (int64_t)r.u64();
        t.elements = e;
        t.bytes = gguf_byte_count(t.dtype, e);
        tensors.push_back(t);
    }
    if (r.eof) { err = "unexpected end of GGUF header"; return SLX_EEOF; }
    long pos = ftell(fp_);
    data_offset = (pos + 31L) & ~31L;
    for (size_t i = 0; i < tensors.size(); i++) index_[tensors[i].name] = i;
    arch = get_string("general.architecture");
    name = get_string("general.name");
    embd = get_int(arch + ".embedding_length");
    ctx = get_int(arch + ".context_length");
    heads = get_int(arch + ".attention.head_count");
    layers = get_int(arch + ".block_count");
    ff = get_int(arch + ".feed_forward_length");
    auto tk = meta.find("tokenizer.ggml.tokens");
    n_tokens = (tk != meta.end() && tk->second.type == 9) ? (int)tk->second.array_len : 0;
    bos = get_int("tokenizer.ggml.bos_token_id");
    eos = get_int("tokenizer.ggml.eos_token_id");
    unk = get_int("tokenizer.ggml.unknown_token_id");
    return SLX_OK;
}

const GgufTensor* GgufFile::tensor(const std::string& n) const {
    auto it = index_.find(n);
    return it == index_.end() ? nullptr : &tensors[it->second];
}

int GgufFile::read_raw(const GgufTensor& t, std::vector<uint8_t>& out, std::string& err) const {
    int64_t need = gguf_decode_bytes(t.dtype, t.elements);
    if (need < 0) {
        err = "Dequantization of dtype " + std::to_string(t.dtype) + " is not yet implemented";
        return SLX_EUNSUPPORTED;
    }
    out.resize((size_t)need);
    if (fseek(fp_, data_offset + t.offset, SEEK_SET) != 0) { err = "seek failed"; return SLX_EEOF; }
    size_t got = need ? fread(out.data(), 1, (size_t)need, fp_) : 0;
    if ((int64_t)got != need) {
        err = "Unexpected end of GGUF stream reading " + t.name;
        return SLX_EEOF;
    }
    return SLX_OK;
}

int GgufFile::get_int(const std::string& key, int def) const {
    auto it = meta.find(key);
    if (it == meta.end()) return def;
    switch (it->second.type) {
        case 5: case 11: return (int)it->second.i;
        case 4: return (int)(uint32_t)it->second.u;
        case 10: return (int)it->second.u;
        default: return 0;
    }
}

int GgufFile::get_int_i32(const std::string& key, int def) const {
    auto it = meta.find(key);
    if (it == meta.end()) return def;
    if (it->second.type == 5) return (int)it->second.i;
    if (it->second.type == 4) return (int)(uint32_t)it->second.u;
    return def;
}

float GgufFile::get_float(const std::string& key, float def) const {
    auto it = meta.find(key);
    if (it == meta.end()) return def;
    if (it->second.type == 6 || it->second.type == 12) return (float)it->second.f;
    return def;
}

std::string GgufFile::get_string(const std::string& key) const {
    auto it = meta.find(key);
    if (it == meta.end() || it->second.type != 8) return "";
    return it->second.s;
}

}  // namespace slx
