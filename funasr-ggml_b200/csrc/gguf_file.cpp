// GGUF model files for the decoder: geometry from the metadata, decoder tensors
// straight from the mapped file into fa_load_weights.
//
// Replaces, for the decoder, the reference's file path:
//   core/gguf_reader.hpp              GGUFReader (gguf_init_from_file, tensor lookup)
//   core/config.hpp:191-228           ModelConfig::load_from_gguf, FunAsr.* keys
//   model/loader.cpp:91-117,210-227   ModelLoader::load_llm / load_llm_layer (llm.* names)
// The reference reads files through ggml's gguf.h, which is not available here; this
// is a reader of its own for the published GGUF container layout (version 2 and 3):
//   magic "GGUF" | u32 version | u64 n_tensors | u64 n_kv
//   n_kv x  (string key, u32 type, value)          string = u64 length + bytes
//   n_tensors x (string name, u32 n_dims, u64 ne[n_dims], u32 ggml type, u64 offset)
//   padding to `general.alignment` (default 32), then the tensor data; each
//   tensor's offset is relative to the start of that data block.
// Every read is bounds-checked against the file size; a malformed file is an error,
// never a read past the mapping.
#include "funasr_dec.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

namespace fa {
int report_op_error(int code, const char* msg);                      // fa_api.cu
int report_ctx_error(const fa_ctx* ctx, int code, const char* msg);  // fa_api.cu
}

namespace {

enum : uint32_t {
    kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7, kStr = 8, kArr = 9,
    kU64 = 10, kI64 = 11, kF64 = 12
};

struct Value {
    uint32_t type = 0;
    double num = 0;           // every scalar as a double (exact for the integers used here)
    uint64_t arr_len = 0;     // arrays: element count
    std::string str;
};

struct Tensor {
    std::string name;
    uint32_t type = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    uint32_t n_dims = 0;
    uint64_t offset = 0;
    size_t nbytes = 0;
};

struct File {
    int fd = -1;
    const uint8_t* base = nullptr;
    size_t size = 0;
    std::unordered_map<std::string, Value> kv;
    std::vector<Tensor> tensors;
    size_t data_start = 0;
    std::string err;

    ~File() {
        if (base) munmap(const_cast<uint8_t*>(base), size);
        if (fd >= 0) close(fd);
    }
};

class Cursor {
public:
    Cursor(const uint8_t* p, size_t n) : p_(p), n_(n) {}
    bool take(void* dst, size_t k) {
        if (k > n_ - off_) return false;
        std::memcpy(dst, p_ + off_, k);
        off_ += k;
        return true;
    }
    template <typename T>
    bool get(T& v) { return take(&v, sizeof(T)); }
    bool str(std::string& s) {
        uint64_t len;
        if (!get(len) || len > n_ - off_) return false;
        s.assign(reinterpret_cast<const char*>(p_ + off_), (size_t)len);
        off_ += (size_t)len;
        return true;
    }
    bool skip(uint64_t k) {
        if (k > n_ - off_) return false;
        off_ += (size_t)k;
        return true;
    }
    size_t off() const { return off_; }

private:
    const uint8_t* p_;
    size_t n_;
    size_t off_ = 0;
};

size_t scalar_size(uint32_t t) {
    switch (t) {
        case kU8: case kI8: case kBool: return 1;
        case kU16: case kI16: return 2;
        case kU32: case kI32: case kF32: return 4;
        case kU64: case kI64: case kF64: return 8;
        default: return 0;
    }
}

bool read_scalar(Cursor& c, uint32_t t, double& out) {
    switch (t) {
        case kU8: { uint8_t v; if (!c.get(v)) return false; out = v; return true; }
        case kI8: { int8_t v; if (!c.get(v)) return false; out = v; return true; }
        case kBool: { uint8_t v; if (!c.get(v)) return false; out = v ? 1 : 0; return true; }
        case kU16: { uint16_t v; if (!c.get(v)) return false; out = v; return true; }
        case kI16: { int16_t v; if (!c.get(v)) return false; out = v; return true; }
        case kU32: { uint32_t v; if (!c.get(v)) return false; out = v; return true; }
        case kI32: { int32_t v; if (!c.get(v)) return false; out = v; return true; }
        case kF32: { float v; if (!c.get(v)) return false; out = v; return true; }
        case kU64: { uint64_t v; if (!c.get(v)) return false; out = (double)v; return true; }
        case kI64: { int64_t v; if (!c.get(v)) return false; out = (double)v; return true; }
        case kF64: { double v; if (!c.get(v)) return false; out = v; return true; }
        default: return false;
    }
}

// Bytes of a tensor of ggml type t with ne0 x rows elements; 0 for types the decoder does not take.
size_t tensor_bytes(uint32_t t, int64_t ne0, int64_t rows) {
    switch (t) {
        case FA_TYPE_F32: return (size_t)ne0 * rows * 4;
        case FA_TYPE_F16: case FA_TYPE_BF16: return (size_t)ne0 * rows * 2;
        case FA_TYPE_Q8_0: return ne0 % 32 ? 0 : (size_t)(ne0 / 32) * 34 * rows;
        default: return 0;
    }
}

bool open_gguf(const char* path, File& f) {
    f.fd = open(path, O_RDONLY);
    if (f.fd < 0) { f.err = std::string("cannot open ") + path; return false; }
    struct stat st;
    if (fstat(f.fd, &st) != 0 || st.st_size < 24) { f.err = std::string(path) + ": not a GGUF file"; return false; }
    f.size = (size_t)st.st_size;
    void* m = mmap(nullptr, f.size, PROT_READ, MAP_PRIVATE, f.fd, 0);
    if (m == MAP_FAILED) { f.err = std::string("cannot map ") + path; return false; }
    f.base = static_cast<const uint8_t*>(m);
    Cursor c(f.base, f.size);
    char magic[4];
    uint32_t version;
    uint64_t n_tensors, n_kv;
    if (!c.take(magic, 4) || std::memcmp(magic, "GGUF", 4) != 0) { f.err = std::string(path) + ": bad magic"; return false; }
    if (!c.get(version) || (version != 2 && version != 3)) {
        f.err = std::string(path) + ": unsupported GGUF version";
        return false;
    }
    if (!c.get(n_tensors) || !c.get(n_kv) || n_tensors > (1u << 24) || n_kv > (1u << 24)) {
        f.err = std::string(path) + ": bad header counts";
        return false;
    }
    for (uint64_t i = 0; i < n_kv; ++i) {
        std::string key;
        Value v;
        if (!c.str(key) || !c.get(v.type)) { f.err = "truncated metadata"; return false; }
        if (v.type == kStr) {
            if (!c.str(v.str)) { f.err = "truncated string value of " + key; return false; }
        } else if (v.type == kArr) {
            uint32_t et;
            if (!c.get(et) || !c.get(v.arr_len)) { f.err = "truncated array header of " + key; return false; }
            if (et == kStr) {
                for (uint64_t j = 0; j < v.arr_len; ++j) {
                    uint64_t len;
                    if (!c.get(len) || !c.skip(len)) { f.err = "truncated string array " + key; return false; }
                }
            } else {
                const size_t es = scalar_size(et);
                if (!es || v.arr_len > f.size || !c.skip(v.arr_len * es)) {
                    f.err = "bad array " + key;
                    return false;
                }
            }
        } else if (!read_scalar(c, v.type, v.num)) {
            f.err = "bad value type of " + key;
            return false;
        }
        f.kv[key] = std::move(v);
    }
    f.tensors.resize((size_t)n_tensors);
    for (auto& t : f.tensors) {
        if (!c.str(t.name) || !c.get(t.n_dims) || t.n_dims < 1 || t.n_dims > 4) {
            f.err = "bad tensor info";
            return false;
        }
        for (uint32_t d = 0; d < t.n_dims; ++d) {
            uint64_t ne;
            if (!c.get(ne) || ne == 0 || ne > (1ull << 40)) { f.err = "bad shape of " + t.name; return false; }
            t.ne[d] = (int64_t)ne;
        }
        if (!c.get(t.type) || !c.get(t.offset)) { f.err = "truncated tensor info of " + t.name; return false; }
    }
    uint64_t align = 32;
    auto it = f.kv.find("general.alignment");
    if (it != f.kv.end() && it->second.type != kStr && it->second.type != kArr) align = (uint64_t)it->second.num;
    if (align == 0 || (align & (align - 1))) { f.err = "bad general.alignment"; return false; }
    f.data_start = (c.off() + align - 1) / align * align;
    for (auto& t : f.tensors) {
        const int64_t rows = t.ne[1] * t.ne[2] * t.ne[3];
        t.nbytes = tensor_bytes(t.type, t.ne[0], rows);
        if (t.nbytes && (t.offset > f.size || f.data_start + t.offset + t.nbytes > f.size)) {
            f.err = t.name + ": data beyond the end of the file";
            return false;
        }
    }
    return true;
}

bool u32_key(const File& f, const char* key, int& out, bool required, std::string& err) {
    auto it = f.kv.find(key);
    if (it == f.kv.end() || it->second.type == kStr || it->second.type == kArr) {
        if (required) err = std::string("missing metadata key ") + key;
        return !required;
    }
    out = (int)it->second.num;
    return true;
}

}  // namespace

extern "C" int fa_gguf_read_desc(const char* path, fa_model_desc* desc) {
    if (!path || !desc) return fa::report_op_error(FA_ERR_INVALID_ARG, "fa_gguf_read_desc: NULL argument");
    File f;
    if (!open_gguf(path, f)) return fa::report_op_error(FA_ERR_WEIGHTS, f.err.c_str());
    fa_model_desc d = *desc;
    std::string err;
    // the keys ModelConfig::load_from_gguf requires, then the optional ones with their defaults
    if (!u32_key(f, "FunAsr.block_count", d.n_layers, true, err) ||
        !u32_key(f, "FunAsr.embedding_length", d.hidden, true, err) ||
        !u32_key(f, "FunAsr.context_length", d.max_ctx, true, err) ||
        !u32_key(f, "FunAsr.feed_forward_length", d.ffn, true, err) ||
        !u32_key(f, "FunAsr.attention.head_count", d.n_heads, true, err) ||
        !u32_key(f, "FunAsr.attention.head_count_kv", d.n_kv_heads, true, err))
        return fa::report_op_error(FA_ERR_WEIGHTS, (std::string(path) + ": " + err).c_str());
    d.head_dim = 128;
    u32_key(f, "FunAsr.attention.key_length", d.head_dim, false, err);
    d.rope_base = 1000000.0f;
    auto it = f.kv.find("FunAsr.rope.freq_base");
    if (it != f.kv.end() && it->second.type != kStr && it->second.type != kArr) d.rope_base = (float)it->second.num;
    // the reference fixes vocab_size at 151936 (core/config.hpp:225); a file's lm_head says the same
    d.vocab = 151936;
    for (const auto& t : f.tensors)
        if (t.name == "llm.lm_head.weight" && t.n_dims >= 2) d.vocab = (int)t.ne[1];
    *desc = d;
    return FA_OK;
}

extern "C" int fa_gguf_find_tensor(const char* path, const char* name, int* type, int64_t* ne, size_t* file_offset,
                                   size_t* nbytes) {
    if (!path || !name) return fa::report_op_error(FA_ERR_INVALID_ARG, "fa_gguf_find_tensor: NULL argument");
    File f;
    if (!open_gguf(path, f)) return fa::report_op_error(FA_ERR_WEIGHTS, f.err.c_str());
    for (const auto& t : f.tensors) {
        if (t.name != name) continue;
        if (type) *type = (int)t.type;
        if (ne) { ne[0] = t.ne[0]; ne[1] = t.ne[1] * t.ne[2] * t.ne[3]; }
        if (file_offset) *file_offset = f.data_start + t.offset;
        if (nbytes) *nbytes = t.nbytes;
        return FA_OK;
    }
    return fa::report_op_error(FA_ERR_WEIGHTS, (std::string(path) + ": no tensor " + name).c_str());
}

extern "C" int fa_load_gguf(fa_ctx* ctx, const char* path) {
    if (!ctx || !path) return fa::report_ctx_error(ctx, FA_ERR_INVALID_ARG, "fa_load_gguf: NULL argument");
    File f;
    if (!open_gguf(path, f)) return fa::report_ctx_error(ctx, FA_ERR_WEIGHTS, f.err.c_str());
    std::vector<fa_tensor_view> views;
    for (const auto& t : f.tensors) {
        if (t.name.compare(0, 4, "llm.") != 0 || !t.nbytes) continue;
        fa_tensor_view v{};
        v.name = t.name.c_str();
        v.type = (int)t.type;
        v.ne[0] = t.ne[0];
        v.ne[1] = t.ne[1] * t.ne[2] * t.ne[3];
        v.data = f.base + f.data_start + t.offset;
        v.nbytes = t.nbytes;
        views.push_back(v);
    }
    return fa_load_weights(ctx, views.data(), (int)views.size());
}
