// GGUF header parser and ConfigFrom.  See gguf.hpp.
#include "gguf.hpp"

#include <algorithm>
#include <climits>
#include <cstring>

namespace llmb {

namespace {

// Bounds, gguf/gguf.go:18-26.
constexpr uint64_t kMaxTensors = 1ull << 16;
constexpr uint64_t kMaxKV = 1ull << 16;
constexpr uint64_t kMaxString = 1ull << 24;
constexpr uint64_t kMaxArray = 1ull << 22;
constexpr uint64_t kMaxHeader = 256ull << 20;
constexpr uint32_t kMaxDims = 4;
constexpr uint64_t kMaxAlignment = 1ull << 20;
constexpr uint64_t kReadAhead = 1ull << 20;  // gguf/gguf.go:145

// Metadata value types, gguf/gguf.go:39-54.
enum : uint32_t { U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 };

// The bounded reader with a read-ahead window, gguf/gguf.go:133-179.
struct Reader {
    const ReadAt &r;
    uint64_t pos = 0, lim = 0;
    std::vector<uint8_t> win;
    uint64_t win_off = 0;

    GgufErr read(void *p, uint64_t n) {
        if (pos + n > lim) return GgufErr::Bound;
        if (n >= kReadAhead) {
            if (r(pos, p, n) < n) return GgufErr::Eof;
            pos += n;
            return GgufErr::Ok;
        }
        if (pos < win_off || pos + n > win_off + win.size()) {
            uint64_t want = std::min(kReadAhead, lim - pos);
            win.resize(want);
            uint64_t got = r(pos, win.data(), want);
            win.resize(got);
            win_off = pos;
            if (got < n) return GgufErr::Eof;
        }
        std::memcpy(p, win.data() + (pos - win_off), n);
        pos += n;
        return GgufErr::Ok;
    }
    GgufErr u32(uint32_t &v) {
        uint8_t b[4];
        GgufErr e = read(b, 4);
        v = uint32_t(b[0]) | uint32_t(b[1]) << 8 | uint32_t(b[2]) << 16 | uint32_t(b[3]) << 24;
        return e;
    }
    GgufErr u64(uint64_t &v) {
        uint32_t lo = 0, hi = 0;
        GgufErr e = u32(lo);
        if (e != GgufErr::Ok) return e;
        e = u32(hi);
        v = uint64_t(hi) << 32 | lo;
        return e;
    }
    // reader.str, gguf/gguf.go:195-208
    GgufErr str(std::string &s) {
        uint64_t n;
        GgufErr e = u64(n);
        if (e != GgufErr::Ok) return e;
        if (n > kMaxString) return GgufErr::Bound;
        if (pos + n > lim) return GgufErr::Bound;
        s.resize(n);
        return read(s.data(), n);
    }
    // reader.value, gguf/gguf.go:210-289
    GgufErr value(uint32_t t, int depth, Value &v) {
        GgufErr e;
        switch (t) {
        case U8: case I8: case BOOL: {
            uint8_t b;
            if ((e = read(&b, 1)) != GgufErr::Ok) return e;
            if (t == U8) v.kind = Value::Uint, v.u = b;
            else if (t == I8) v.kind = Value::Int, v.i = int8_t(b);
            else v.kind = Value::Bool, v.b = b != 0;
            return GgufErr::Ok;
        }
        case U16: case I16: {
            uint8_t b[2];
            if ((e = read(b, 2)) != GgufErr::Ok) return e;
            uint16_t x = uint16_t(b[0] | b[1] << 8);
            if (t == U16) v.kind = Value::Uint, v.u = x;
            else v.kind = Value::Int, v.i = int16_t(x);
            return GgufErr::Ok;
        }
        case U32: case I32: case F32: {
            uint32_t x;
            if ((e = u32(x)) != GgufErr::Ok) return e;
            if (t == U32) v.kind = Value::Uint, v.u = x;
            else if (t == I32) v.kind = Value::Int, v.i = int32_t(x);
            else {
                float f;
                std::memcpy(&f, &x, 4);
                v.kind = Value::Float, v.f = f;
            }
            return GgufErr::Ok;
        }
        case U64: case I64: case F64: {
            uint64_t x;
            if ((e = u64(x)) != GgufErr::Ok) return e;
            if (t == U64) v.kind = Value::Uint, v.u = x;
            else if (t == I64) v.kind = Value::Int, v.i = int64_t(x);
            else std::memcpy(&v.f, &x, 8), v.kind = Value::Float;
            return GgufErr::Ok;
        }
        case STRING:
            v.kind = Value::String;
            return str(v.s);
        case ARRAY: {
            if (depth > 0) return GgufErr::Format;
            uint32_t et;
            uint64_t n;
            if ((e = u32(et)) != GgufErr::Ok) return e;
            if ((e = u64(n)) != GgufErr::Ok) return e;
            if (n > kMaxArray) return GgufErr::Bound;
            if (n > lim - pos) return GgufErr::Bound;  // gguf/gguf.go:273-277
            for (uint64_t i = 0; i < n; i++) {
                Value el;
                if ((e = value(et, depth + 1, el)) != GgufErr::Ok) return e;
            }
            v.kind = Value::Array, v.n = n;
            return GgufErr::Ok;
        }
        }
        return GgufErr::Format;
    }
};

const char *err_name(GgufErr e) {
    switch (e) {
    case GgufErr::Magic: return "gguf: bad magic";
    case GgufErr::Version: return "gguf: unsupported version";
    case GgufErr::Bound: return "gguf: a size or count exceeds its bound";
    case GgufErr::Format: return "gguf: malformed header";
    case GgufErr::Eof: return "gguf: unexpected end of file";
    case GgufErr::Io: return "gguf: read error";
    default: return "gguf: ok";
    }
}

}  // namespace

bool block_size(uint32_t type, uint64_t &elems, uint64_t &bytes) {
    switch (type) {
    case GGML_F32: elems = 1, bytes = 4; return true;
    case GGML_F16: elems = 1, bytes = 2; return true;
    case GGML_Q4_0: elems = 32, bytes = 18; return true;
    case GGML_Q4_1: elems = 32, bytes = 20; return true;
    case GGML_Q5_0: elems = 32, bytes = 22; return true;
    case GGML_Q5_1: elems = 32, bytes = 24; return true;
    case GGML_Q8_0: elems = 32, bytes = 34; return true;
    case GGML_Q6_K: elems = 256, bytes = 210; return true;
    }
    elems = bytes = 0;
    return false;
}

const Tensor *GgufFile::tensor(const std::string &name) const {
    auto it = by_name.find(name);
    return it == by_name.end() ? nullptr : &tensors[it->second];
}

bool GgufFile::get_uint(const std::string &key, uint64_t &v) const {  // gguf/gguf.go:410-420
    v = 0;
    auto it = meta.find(key);
    if (it == meta.end()) return false;
    if (it->second.kind == Value::Uint) return v = it->second.u, true;
    if (it->second.kind == Value::Int && it->second.i >= 0) return v = uint64_t(it->second.i), true;
    return false;
}

bool GgufFile::get_float(const std::string &key, double &v) const {  // gguf/gguf.go:423-426
    v = 0;
    auto it = meta.find(key);
    if (it == meta.end() || it->second.kind != Value::Float) return false;
    v = it->second.f;
    return true;
}

bool GgufFile::get_str(const std::string &key, std::string &v) const {  // gguf/gguf.go:429-432
    auto it = meta.find(key);
    if (it == meta.end() || it->second.kind != Value::String) return false;
    v = it->second.s;
    return true;
}

GgufErr gguf_parse(const ReadAt &ra, uint64_t size, GgufFile &f, std::string &err) {
    Reader r{ra};
    r.lim = std::min(size, kMaxHeader);
    auto fail = [&](GgufErr e, const std::string &what) {
        err = std::string(err_name(e)) + (what.empty() ? "" : ": " + what);
        return e;
    };
    char magic[4];
    GgufErr e;
    if ((e = r.read(magic, 4)) != GgufErr::Ok) return fail(e, "");
    if (std::memcmp(magic, "GGUF", 4) != 0) return fail(GgufErr::Magic, "");
    uint32_t ver;
    if ((e = r.u32(ver)) != GgufErr::Ok) return fail(e, "");
    if (ver != 3) return fail(GgufErr::Version, std::to_string(ver));
    uint64_t nt, nkv;
    if ((e = r.u64(nt)) != GgufErr::Ok || (e = r.u64(nkv)) != GgufErr::Ok) return fail(e, "");
    if (nt > kMaxTensors || nkv > kMaxKV)
        return fail(GgufErr::Bound, std::to_string(nt) + " tensors, " + std::to_string(nkv) + " metadata entries");
    f = GgufFile{};
    f.version = ver;
    f.size = size;
    for (uint64_t i = 0; i < nkv; i++) {
        std::string k;
        uint32_t t;
        Value v;
        if ((e = r.str(k)) != GgufErr::Ok || (e = r.u32(t)) != GgufErr::Ok) return fail(e, "");
        if ((e = r.value(t, 0, v)) != GgufErr::Ok) return fail(e, "key \"" + k + "\"");
        f.meta[k] = std::move(v);
    }
    f.alignment = 32;
    auto a = f.meta.find("general.alignment");
    if (a != f.meta.end()) {
        const Value &v = a->second;
        if (v.kind != Value::Uint || v.u == 0 || v.u > kMaxAlignment || v.u % 8 != 0)
            return fail(GgufErr::Format, "general.alignment");
        f.alignment = v.u;
    }
    f.tensors.reserve(std::min<uint64_t>(nt, 1024));
    for (uint64_t i = 0; i < nt; i++) {
        Tensor t;
        uint32_t nd;
        if ((e = r.str(t.name)) != GgufErr::Ok || (e = r.u32(nd)) != GgufErr::Ok) return fail(e, "");
        if (nd == 0 || nd > kMaxDims)
            return fail(GgufErr::Format, "tensor \"" + t.name + "\" has " + std::to_string(nd) + " dimensions");
        t.dims.resize(nd);
        uint64_t elems = 1;
        for (uint32_t j = 0; j < nd; j++) {
            uint64_t d;
            if ((e = r.u64(d)) != GgufErr::Ok) return fail(e, "");
            if (d == 0 || d > (1ull << 32)) return fail(GgufErr::Bound, "tensor \"" + t.name + "\" dimension");
            if (elems > (1ull << 62) / d) return fail(GgufErr::Bound, "tensor \"" + t.name + "\" too large");
            elems *= d;
            t.dims[j] = d;
        }
        if ((e = r.u32(t.type)) != GgufErr::Ok || (e = r.u64(t.offset)) != GgufErr::Ok) return fail(e, "");
        uint64_t be, bb;
        if (!block_size(t.type, be, bb))
            return fail(GgufErr::Format, "tensor \"" + t.name + "\" has unsupported ggml type " + std::to_string(t.type));
        if (t.dims[0] % be != 0) return fail(GgufErr::Format, "tensor \"" + t.name + "\" row is not whole blocks");
        t.size = elems / be * bb;
        if (f.by_name.count(t.name)) return fail(GgufErr::Format, "duplicate tensor \"" + t.name + "\"");
        f.by_name[t.name] = f.tensors.size();
        f.tensors.push_back(std::move(t));
    }
    f.data_offset = (r.pos + f.alignment - 1) / f.alignment * f.alignment;
    for (const Tensor &t : f.tensors) {
        if (t.offset % f.alignment != 0) return fail(GgufErr::Format, "tensor \"" + t.name + "\" offset is not aligned");
        if (t.offset > size || f.data_offset > size - t.offset || t.size > size - f.data_offset - t.offset)
            return fail(GgufErr::Bound, "tensor \"" + t.name + "\" lies past the end of the file");
    }
    return GgufErr::Ok;
}

bool config_from(const GgufFile &f, Config &c, std::string &err) {
    c = Config{};
    std::string arch;
    f.get_str("general.architecture", arch);
    if (arch != "llama" && arch != "qwen2") {
        err = "llm: architecture \"" + arch + "\" is not supported (llama and qwen2 only)";
        return false;
    }
    auto u = [&](const char *k) {
        uint64_t v;
        f.get_uint(arch + "." + k, v);
        return int64_t(v);
    };
    int64_t layers = u("block_count"), embd = u("embedding_length"), ff = u("feed_forward_length");
    int64_t heads = u("attention.head_count"), kvh = u("attention.head_count_kv"), ctx = u("context_length");
    if (kvh == 0) kvh = heads;
    if (layers <= 0 || embd <= 0 || ff <= 0 || heads <= 0 || kvh <= 0 || embd % heads != 0 || heads % kvh != 0 ||
        layers > INT_MAX || embd > INT_MAX || ff > INT_MAX || ctx < 0 || ctx > INT_MAX) {
        err = "llm: implausible " + arch + " hyperparameters";
        return false;
    }
    c.arch = arch;
    c.rope_neox = arch == "qwen2";
    c.layers = int(layers), c.embd = int(embd), c.ff = int(ff), c.heads = int(heads), c.kv_heads = int(kvh);
    c.ctx = int(ctx);
    c.head_dim = c.embd / c.heads;
    int64_t rd = u("rope.dimension_count");
    if (rd != 0 && rd != c.head_dim) {
        err = "llm: rope.dimension_count " + std::to_string(rd) + " differs from the head size " + std::to_string(c.head_dim);
        return false;
    }
    for (const char *k : {".rope.scaling.type", ".rope.scaling.factor"})
        if (f.meta.count(arch + k)) {
            err = "llm: rope scaling (" + arch + k + ") is not supported";
            return false;
        }
    double rb, eps;
    if (!f.get_float(arch + ".rope.freq_base", rb)) rb = 10000;
    f.get_float(arch + ".attention.layer_norm_rms_epsilon", eps);
    c.rope_base = float(rb), c.eps = float(eps);
    const Tensor *te = f.tensor("token_embd.weight");
    if (!te) {
        err = "llm: no token_embd.weight";
        return false;
    }
    if (te->dims.size() < 2 || te->dims[1] > INT_MAX) {  // config.go:62 would panic on a vector
        err = "llm: token_embd.weight is not a matrix";
        return false;
    }
    c.vocab = int(te->dims[1]);
    c.tied_output = f.tensor("output.weight") == nullptr;
    c.bias = f.tensor("blk.0.attn_q.bias") != nullptr;
    if (c.bias != (arch == "qwen2")) {
        err = "llm: " + arch + " with biases " + (c.bias ? "true" : "false") + " is not supported";
        return false;
    }
    return true;
}

float f16_to_f32(uint16_t h) {
    uint32_t sign = uint32_t(h >> 15) << 31, exp = (uint32_t(h) >> 10) & 0x1f, man = uint32_t(h) & 0x3ff, bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            uint32_t e = 127 - 15 + 1;
            while ((man & 0x400) == 0) man <<= 1, e--;
            bits = sign | e << 23 | (man & 0x3ff) << 13;
        }
    } else if (exp == 31) {
        bits = sign | 0xffu << 23 | man << 13;
    } else {
        bits = sign | (exp + 127 - 15) << 23 | man << 13;
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

}  // namespace llmb
