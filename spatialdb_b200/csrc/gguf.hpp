// gguf.hpp -- host-side GGUF container reader for libslx.
//
// Parses what GgufReader parses (SparseLattice/Gguf/GgufReader.cs:54-130): magic 0x46554747,
// version 2 or 3, metadata key/values (GgufReader.cs:214-243), the tensor table
// (name, dims as u64 truncated to int, dtype u32, offset u64) and a data section that starts at
// the next 32-byte boundary after the table (GgufReader.cs:99-101; general.alignment is ignored,
// as in the reference). Tensor bytes are read on demand.
#pragma once
#include <cstdint>
#include <cstdio>
#include <map>
#include <string>
#include <vector>

namespace slx {

enum GgufDType : uint32_t {
    GG_F32 = 0, GG_F16 = 1, GG_Q4_0 = 2, GG_Q4_1 = 3, GG_Q5_0 = 6, GG_Q5_1 = 7, GG_Q8_0 = 8,
    GG_Q2_K = 10, GG_Q3_K = 11, GG_Q4_K = 12, GG_Q5_K = 13, GG_Q6_K = 14, GG_Q8_K = 15,
    GG_BF16 = 30, GG_MXFP4 = 39,
};

struct GgufValue {
    uint32_t type = 0;
    int64_t i = 0;
    uint64_t u = 0;
    double f = 0;
    std::string s;
    uint64_t array_len = 0;
    uint32_t array_type = 0;
};

struct GgufTensor {
    std::string name;
    std::vector<int> shape;
    uint32_t dtype = 0;
    int64_t offset = 0;
    int64_t elements = 0;
    int64_t bytes = 0;
};

int64_t gguf_byte_count(uint32_t dtype, int64_t elements);   // GgufTensorInfo.cs:27-48
int64_t gguf_decode_bytes(uint32_t dtype, int64_t elements); // bytes GgufDequantizer consumes, -1 if undecodable

class GgufFile {
public:
    // status: 0 ok, else an SLX_* error code; err receives a message.
    int open(const std::string& path, std::string& err);
    ~GgufFile();

    const GgufTensor* tensor(const std::string& name) const;
    // Reads the bytes the reference's dequantizer would read for this tensor.
    int read_raw(const GgufTensor& t, std::vector<uint8_t>& out, std::string& err) const;

    int get_int(const std::string& key, int def = 0) const;        // GgufReader.GetInt semantics (:252-263)
    int get_int_i32(const std::string& key, int def) const;        // *Source.GetInt: Int32/UInt32 only
    float get_float(const std::string& key, float def) const;      // *Source.GetFloat: Float32/Float64 only
    std::string get_string(const std::string& key) const;

    uint32_t version = 0;
    int64_t data_offset = 0;
    std::string arch, name;
    int embd = 0, ctx = 0, heads = 0, layers = 0, ff = 0;
    int n_tokens = 0, bos = 0, eos = 0, unk = 0;
    std::map<std::string, GgufValue> meta;
    std::vector<GgufTensor> tensors;

private:
    FILE* fp_ = nullptr;
    std::map<std::string, size_t> index_;
};

}  // namespace slx
