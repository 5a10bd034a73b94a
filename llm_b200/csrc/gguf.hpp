// GGUF v3 header parser and model configuration (host side of the loader).
//
// Restates the reference's bounded parser, gguf/gguf.go:18-432, and
// ConfigFrom, config.go:29-73.  The header is read through a callback with a
// read-ahead window (gguf/gguf.go:142-179); tensor data is never read here.
#pragma once

#include <cstdint>
#include <functional>
#include <string>
#include <unordered_map>
#include <vector>

namespace llmb {

// ggml tensor types, gguf/gguf.go:59-69.
enum GgmlType : uint32_t {
    GGML_F32 = 0,
    GGML_F16 = 1,
    GGML_Q4_0 = 2,
    GGML_Q4_1 = 3,
    GGML_Q5_0 = 6,
    GGML_Q5_1 = 7,
    GGML_Q8_0 = 8,
    GGML_Q6_K = 14,
};

// Type.BlockSize, gguf/gguf.go:72-92.
bool block_size(uint32_t type, uint64_t &elems, uint64_t &bytes);

// Error classes of gguf/gguf.go:29-34 (plus a short read).
enum class GgufErr { Ok = 0, Magic, Version, Bound, Format, Eof, Io };

struct Tensor {  // gguf/gguf.go:96-102
    std::string name;
    std::vector<uint64_t> dims;  // ne[0] first (contiguous)
    uint32_t type = 0;
    uint64_t offset = 0, size = 0;
};

// A metadata value, as Go keeps it (gguf/gguf.go:116).
struct Value {
    enum Kind { None, Uint, Int, Float, Bool, String, Array } kind = None;
    uint64_t u = 0;
    int64_t i = 0;
    double f = 0;
    bool b = false;
    std::string s;
    uint64_t n = 0;  // array length
};

// Reads len bytes at offset into buf; returns the number of bytes read.
using ReadAt = std::function<uint64_t(uint64_t offset, void *buf, uint64_t len)>;

struct GgufFile {  // gguf/gguf.go:113-122
    uint32_t version = 0;
    std::unordered_map<std::string, Value> meta;
    std::vector<Tensor> tensors;
    std::unordered_map<std::string, size_t> by_name;
    uint64_t data_offset = 0, alignment = 32, size = 0;

    const Tensor *tensor(const std::string &name) const;
    bool get_uint(const std::string &key, uint64_t &v) const;  // File.Uint
    bool get_float(const std::string &key, double &v) const;   // File.Float
    bool get_str(const std::string &key, std::string &v) const;  // File.Str
};

// Parse, gguf/gguf.go:291-407.  On failure returns the error class and a
// message in err.
GgufErr gguf_parse(const ReadAt &r, uint64_t size, GgufFile &out, std::string &err);

// Config, config.go:11-23.
struct Config {
    int layers = 0, embd = 0, ff = 0, heads = 0, kv_heads = 0, head_dim = 0, vocab = 0, ctx = 0;
    float rope_base = 0, eps = 0;
    std::string arch;
    bool rope_neox = false, bias = false, tied_output = false;
};

// ConfigFrom, config.go:29-73.  Returns false with a message.
bool config_from(const GgufFile &f, Config &c, std::string &err);

// binary16 -> float32, exact (F16ToF32, f16.go:6-28).
float f16_to_f32(uint16_t h);

}  // namespace llmb
