// jk_gguf.cu -- GGUF reader and weight loader (host code only).
//
// Restates the reference's reader, crates/jevons-formats/src/gguf.rs:
//   limits (strings <= 2^24 bytes, arrays <= 2^26 values, <= 4 dims, <= 2^20 tensors / keys) :12-15, 250-252
//   metadata values (13 kinds, no nested arrays, booleans 0/1, UTF-8 strings)                :186-231
//   Gguf::open: magic, version 2..3, general.alignment (power of two, default 32), tensor
//     infos, data start = header end rounded up to the alignment, per tensor: checked element
//     count, block-aligned rows, bytes, offset aligned and inside the file                     :234-324
//   Value::as_u64 / as_i64 / as_f64 / as_str, Gguf::u64 / f32 / tensor / read / read_range /
//   read_f32                                                                                   :53-105, 326-391
// with the reference's error texts ("Invalid GGUF file: ...", "I/O error reading the model: ...",
// "Missing GGUF metadata key ...", "Missing tensor ..."). Tensor data is read with positional I/O.
// jk_qmatrix_from_gguf is the load path GGUF -> raw blocks -> QMatrix::upload.
#include "jk_internal.h"

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace {

constexpr uint64_t MAX_STRING = 1ull << 24;
constexpr uint64_t MAX_ARRAY = 1ull << 26;
constexpr uint32_t MAX_DIMS = 4;

enum Kind : int {
    K_U8 = 0, K_I8 = 1, K_U16 = 2, K_I16 = 3, K_U32 = 4, K_I32 = 5, K_F32 = 6, K_BOOL = 7,
    K_STRING = 8, K_ARRAY = 9, K_U64 = 10, K_I64 = 11, K_F64 = 12,
};

struct Value {
    int kind = K_U8;
    uint64_t u = 0;  // unsigned kinds and bool
    int64_t i = 0;   // signed kinds
    double f = 0.0;  // f32 (widened) / f64
    std::string s;
    int elem_kind = -1;  // arrays
    std::vector<Value> items;

    bool as_u64(uint64_t* out) const {
        switch (kind) {
        case K_U8: case K_U16: case K_U32: case K_U64: *out = u; return true;
        case K_I8: case K_I16: case K_I32: case K_I64:
            if (i < 0) return false;
            *out = (uint64_t)i;
            return true;
        default: return false;
        }
    }
    bool as_i64(int64_t* out) const {
        switch (kind) {
        case K_I8: case K_I16: case K_I32: case K_I64: *out = i; return true;
        default: {
            uint64_t v;
            if (!as_u64(&v) || v > (uint64_t)INT64_MAX) return false;
            *out = (int64_t)v;
            return true;
        }
        }
    }
    bool as_f64(double* out) const {
        if (kind != K_F32 && kind != K_F64) return false;
        *out = f;
        return true;
    }
};

struct Tensor {
    std::string name;
    std::vector<uint64_t> dims;
    int type = 0;
    bool known = false;  // a type with a block size (TensorType::block)
    uint64_t offset = 0; // absolute
    uint64_t bytes = 0;
};

struct ParseError {
    jk_status st;
    std::string msg;
};

[[noreturn]] void format_err(const std::string& m) { throw ParseError{JK_ERR_INVALID, "Invalid GGUF file: " + m}; }
[[noreturn]] void io_err(const std::string& m) { throw ParseError{JK_ERR_INVALID, "I/O error reading the model: " + m}; }

bool block_of(int type, uint64_t* elems, uint64_t* bytes) {
    switch (type) {
    case JK_TYPE_F32: *elems = 1; *bytes = 4; return true;
    case JK_TYPE_F16: *elems = 1; *bytes = 2; return true;
    case JK_TYPE_Q4_K: *elems = 256; *bytes = 144; return true;
    case JK_TYPE_Q5_0: *elems = 32; *bytes = 22; return true;
    case JK_TYPE_Q6_K: *elems = 256; *bytes = 210; return true;
    case JK_TYPE_Q8_0: *elems = 32; *bytes = 34; return true;
    default: return false;
    }
}

// TensorType's Debug names, as the reference prints them in messages.
std::string type_debug(int type) {
    switch (type) {
    case JK_TYPE_F32: return "F32";
    case JK_TYPE_F16: return "F16";
    case JK_TYPE_Q4_K: return "Q4K";
    case JK_TYPE_Q5_0: return "Q5_0";
    case JK_TYPE_Q6_K: return "Q6K";
    case JK_TYPE_Q8_0: return "Q8_0";
    default: return "Other(" + std::to_string(type) + ")";
    }
}

// Strict UTF-8 (no overlong forms, no surrogates, <= U+10FFFF), as String::from_utf8 requires.
bool valid_utf8(const std::string& s) {
    const auto* p = reinterpret_cast<const unsigned char*>(s.data());
    size_t i = 0, n = s.size();
    while (i < n) {
        const unsigned c = p[i];
        if (c < 0x80) { ++i; continue; }
        int len;
        unsigned cp;
        if ((c & 0xE0) == 0xC0) { len = 2; cp = c & 0x1F; }
        else if ((c & 0xF0) == 0xE0) { len = 3; cp = c & 0x0F; }
        else if ((c & 0xF8) == 0xF0) { len = 4; cp = c & 0x07; }
        else return false;
        if (i + len > n) return false;
        for (int j = 1; j < len; ++j) {
            if ((p[i + j] & 0xC0) != 0x80) return false;
            cp = (cp << 6) | (p[i + j] & 0x3F);
        }
        if ((len == 2 && cp < 0x80) || (len == 3 && cp < 0x800) || (len == 4 && cp < 0x10000)) return false;
        if (cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return false;
        i += len;
    }
    return true;
}

// Buffered sequential reader over the header.
struct Reader {
    FILE* f;
    uint64_t pos = 0;
    void bytes(void* dst, size_t n) {
        if (n && fread(dst, 1, n, f) != n) io_err(ferror(f) ? std::string(strerror(errno)) : "failed to fill whole buffer");
        pos += n;
    }
    uint8_t u8() { uint8_t v; bytes(&v, 1); return v; }
    uint16_t u16() { uint8_t b[2]; bytes(b, 2); return (uint16_t)(b[0] | (b[1] << 8)); }
    uint32_t u32() {
        uint8_t b[4];
        bytes(b, 4);
        return (uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16) | ((uint32_t)b[3] << 24);
    }
    uint64_t u64() { const uint64_t lo = u32(); return lo | ((uint64_t)u32() << 32); }
    std::string string() {
        const uint64_t len = u64();
        if (len > MAX_STRING) format_err("string is too long");
        std::string s(len, '\0');
        bytes(s.data(), len);
        if (!valid_utf8(s)) format_err("string is not UTF-8");
        return s;
    }
    Value value(uint32_t kind, int depth) {
        Value v;
        v.kind = (int)kind;
        switch (kind) {
        case K_U8: v.u = u8(); break;
        case K_I8: v.i = (int8_t)u8(); break;
        case K_U16: v.u = u16(); break;
        case K_I16: v.i = (int16_t)u16(); break;
        case K_U32: v.u = u32(); break;
        case K_I32: v.i = (int32_t)u32(); break;
        case K_F32: { const uint32_t b = u32(); float x; memcpy(&x, &b, 4); v.f = x; break; }
        case K_BOOL: {
            const uint8_t b = u8();
            if (b > 1) format_err("invalid boolean");
            v.u = b;
            break;
        }
        case K_STRING: v.s = string(); break;
        case K_ARRAY: {
            if (depth > 0) format_err("nested arrays are not supported");
            const uint32_t inner = u32();
            const uint64_t len = u64();
            if (len > MAX_ARRAY) format_err("array is too long");
            v.elem_kind = (int)inner;
            v.items.reserve((size_t)len);
            for (uint64_t j = 0; j < len; ++j) v.items.push_back(value(inner, depth + 1));
            break;
        }
        case K_U64: v.u = u64(); break;
        case K_I64: v.i = (int64_t)u64(); break;
        case K_F64: { const uint64_t b = u64(); memcpy(&v.f, &b, 8); break; }
        default: format_err("unknown metadata type " + std::to_string(kind));
        }
        return v;
    }
};

}  // namespace

struct jk_gguf {
    int fd = -1;
    std::map<std::string, Value> metadata;
    std::vector<Tensor> tensors;              // file order
    std::map<std::string, size_t> by_name;
    ~jk_gguf() {
        if (fd >= 0) close(fd);
    }
};

using jk::fail;

namespace {

const Value* find_key(const jk_gguf* g, const char* key) {
    if (!g || !key) return nullptr;
    auto it = g->metadata.find(key);
    return it == g->metadata.end() ? nullptr : &it->second;
}

jk_status missing_key(const char* key) {
    return fail(JK_ERR_INVALID, std::string("Missing GGUF metadata key ") + (key ? key : ""));
}

const Tensor* find_tensor(const jk_gguf* g, const char* name) {
    if (!g || !name) return nullptr;
    auto it = g->by_name.find(name);
    return it == g->by_name.end() ? nullptr : &g->tensors[it->second];
}

jk_status missing_tensor(const char* name) {
    return fail(JK_ERR_INVALID, std::string("Missing tensor ") + (name ? name : ""));
}

void fill_info(const Tensor& t, jk_gguf_tensor_info* out) {
    out->name = t.name.c_str();
    out->n_dims = (uint32_t)t.dims.size();
    for (uint32_t d = 0; d < 4; ++d) out->dims[d] = d < t.dims.size() ? t.dims[d] : 1;
    out->type = t.type;
    out->offset = t.offset;
    out->bytes = t.bytes;
}

jk_status pread_all(int fd, void* dst, uint64_t len, uint64_t offset) {
    auto* p = static_cast<uint8_t*>(dst);
    while (len) {
        const ssize_t r = pread(fd, p, len > (1u << 30) ? (1u << 30) : (size_t)len, (off_t)offset);
        if (r < 0) {
            if (errno == EINTR) continue;
            return fail(JK_ERR_INVALID, std::string("I/O error reading the model: ") + strerror(errno));
        }
        if (r == 0) return fail(JK_ERR_INVALID, "I/O error reading the model: failed to fill whole buffer");
        p += r;
        len -= (uint64_t)r;
        offset += (uint64_t)r;
    }
    return JK_OK;
}

}  // namespace

extern "C" jk_status jk_gguf_open(const char* path, jk_gguf** out) {
    if (!path || !out) return fail(JK_ERR_INVALID, "null pointer");
    *out = nullptr;
    FILE* f = fopen(path, "rb");
    if (!f) return fail(JK_ERR_INVALID, std::string("I/O error reading the model: ") + strerror(errno));
    std::unique_ptr<FILE, int (*)(FILE*)> guard(f, fclose);
    struct stat st;
    if (fstat(fileno(f), &st) != 0) return fail(JK_ERR_INVALID, std::string("I/O error reading the model: ") + strerror(errno));
    const uint64_t file_len = (uint64_t)st.st_size;
    auto g = std::make_unique<jk_gguf>();
    try {
        Reader r{f};
        char magic[4];
        r.bytes(magic, 4);
        if (memcmp(magic, "GGUF", 4) != 0) format_err("bad magic");
        const uint32_t version = r.u32();
        if (version < 2 || version > 3) format_err("unsupported version " + std::to_string(version));
        const uint64_t tensor_count = r.u64();
        const uint64_t kv_count = r.u64();
        if (tensor_count > (1u << 20) || kv_count > (1u << 20)) format_err("implausible header counts");
        for (uint64_t j = 0; j < kv_count; ++j) {
            std::string key = r.string();
            const uint32_t kind = r.u32();
            Value v = r.value(kind, 0);
            if (!g->metadata.emplace(std::move(key), std::move(v)).second) format_err("duplicate metadata key");
        }
        uint64_t alignment = 32;
        if (auto it = g->metadata.find("general.alignment"); it != g->metadata.end()) {
            uint64_t a;
            if (!it->second.as_u64(&a) || a == 0 || (a & (a - 1)) != 0) format_err("invalid alignment");
            alignment = a;
        }
        std::vector<Tensor> infos;
        infos.reserve((size_t)tensor_count);
        for (uint64_t j = 0; j < tensor_count; ++j) {
            Tensor t;
            t.name = r.string();
            const uint32_t n_dims = r.u32();
            if (n_dims == 0 || n_dims > MAX_DIMS)
                format_err("tensor " + t.name + " has " + std::to_string(n_dims) + " dimensions");
            for (uint32_t d = 0; d < n_dims; ++d) t.dims.push_back(r.u64());
            t.type = (int)r.u32();
            t.offset = r.u64();
            infos.push_back(std::move(t));
        }
        const uint64_t header_end = r.pos;
        const uint64_t data_start = (header_end + alignment - 1) / alignment * alignment;
        for (Tensor& t : infos) {
            uint64_t elements = 1;
            for (uint64_t d : t.dims) {
                if (d != 0 && elements > UINT64_MAX / d) format_err("tensor " + t.name + " is too large");
                elements *= d;
            }
            uint64_t be, bb;
            t.known = block_of(t.type, &be, &bb);
            if (t.known) {
                if (t.dims[0] % be != 0) format_err("tensor " + t.name + " rows are not block aligned");
                t.bytes = elements / be * bb;
            }
            const uint64_t start = data_start + t.offset;
            const bool ok = start >= data_start && t.offset % alignment == 0 && start + t.bytes >= start &&
                            start + t.bytes <= file_len;
            if (!ok) format_err("tensor " + t.name + " is out of bounds");
            t.offset = start;
            if (!g->by_name.emplace(t.name, g->tensors.size()).second) format_err("duplicate tensor name");
            g->tensors.push_back(std::move(t));
        }
    } catch (const ParseError& e) {
        return fail(e.st, e.msg);
    }
    g->fd = open(path, O_RDONLY | O_CLOEXEC);
    if (g->fd < 0) return fail(JK_ERR_INVALID, std::string("I/O error reading the model: ") + strerror(errno));
    *out = g.release();
    return JK_OK;
}

extern "C" void jk_gguf_close(jk_gguf* g) { delete g; }

extern "C" size_t jk_gguf_tensor_count(const jk_gguf* g) { return g ? g->tensors.size() : 0; }
extern "C" size_t jk_gguf_metadata_count(const jk_gguf* g) { return g ? g->metadata.size() : 0; }

extern "C" jk_status jk_gguf_tensor_at(const jk_gguf* g, size_t i, jk_gguf_tensor_info* out) {
    if (!g || !out) return fail(JK_ERR_INVALID, "null pointer");
    if (i >= g->tensors.size()) return fail(JK_ERR_INVALID, "tensor index out of range");
    fill_info(g->tensors[i], out);
    return JK_OK;
}

extern "C" jk_status jk_gguf_tensor(const jk_gguf* g, const char* name, jk_gguf_tensor_info* out) {
    if (!g || !out) return fail(JK_ERR_INVALID, "null pointer");
    const Tensor* t = find_tensor(g, name);
    if (!t) return missing_tensor(name);
    fill_info(*t, out);
    return JK_OK;
}

extern "C" jk_status jk_gguf_read(const jk_gguf* g, const char* name, uint64_t start, uint64_t len, void* dst) {
    if (!g) return fail(JK_ERR_INVALID, "null pointer");
    const Tensor* t = find_tensor(g, name);
    if (!t) return missing_tensor(name);
    if (!t->known) return fail(JK_ERR_INVALID, "Invalid GGUF file: tensor " + t->name + " has unsupported type " + type_debug(t->type));
    if (start + len < start || start + len > t->bytes)
        return fail(JK_ERR_INVALID, "Invalid GGUF file: range is outside tensor " + t->name);
    if (len && !dst) return fail(JK_ERR_INVALID, "null destination");
    return pread_all(g->fd, dst, len, t->offset + start);
}

extern "C" jk_status jk_gguf_read_f32(const jk_gguf* g, const char* name, float* dst, size_t dst_len) {
    if (!g) return fail(JK_ERR_INVALID, "null pointer");
    const Tensor* t = find_tensor(g, name);
    if (!t) return missing_tensor(name);
    if (t->type != JK_TYPE_F32) return fail(JK_ERR_INVALID, "Invalid GGUF file: tensor " + t->name + " is not F32");
    if (dst_len < t->bytes / 4) return fail(JK_ERR_INVALID, "read_f32: destination too small");
    return jk_gguf_read(g, name, 0, t->bytes, dst);
}

extern "C" jk_status jk_gguf_value_kind(const jk_gguf* g, const char* key, int* kind, int* elem_kind, size_t* len) {
    const Value* v = find_key(g, key);
    if (!v) return missing_key(key);
    if (kind) *kind = v->kind;
    if (elem_kind) *elem_kind = v->kind == K_ARRAY ? v->elem_kind : -1;
    if (len) *len = v->kind == K_ARRAY ? v->items.size() : v->kind == K_STRING ? v->s.size() : 1;
    return JK_OK;
}

namespace {

// The value at `key`, or element `index` of the array at `key` when index >= 0.
jk_status value_at(const jk_gguf* g, const char* key, int64_t index, const Value** out) {
    const Value* v = find_key(g, key);
    if (!v) return missing_key(key);
    if (index >= 0) {
        if (v->kind != K_ARRAY) return fail(JK_ERR_INVALID, std::string("Invalid GGUF file: ") + key + " is not an array");
        if ((uint64_t)index >= v->items.size()) return fail(JK_ERR_INVALID, std::string("array index out of range for ") + key);
        v = &v->items[(size_t)index];
    }
    *out = v;
    return JK_OK;
}

}  // namespace

extern "C" jk_status jk_gguf_u64(const jk_gguf* g, const char* key, int64_t index, uint64_t* out) {
    const Value* v;
    if (jk_status st = value_at(g, key, index, &v)) return st;
    if (!out || !v->as_u64(out)) return fail(JK_ERR_INVALID, std::string("Invalid GGUF file: ") + key + " is not an unsigned integer");
    return JK_OK;
}

extern "C" jk_status jk_gguf_i64(const jk_gguf* g, const char* key, int64_t index, int64_t* out) {
    const Value* v;
    if (jk_status st = value_at(g, key, index, &v)) return st;
    if (!out || !v->as_i64(out)) return fail(JK_ERR_INVALID, std::string("Invalid GGUF file: ") + key + " is not an integer");
    return JK_OK;
}

extern "C" jk_status jk_gguf_f32(const jk_gguf* g, const char* key, int64_t index, float* out) {
    const Value* v;
    if (jk_status st = value_at(g, key, index, &v)) return st;
    double d;
    if (!out || !v->as_f64(&d)) return fail(JK_ERR_INVALID, std::string("Invalid GGUF file: ") + key + " is not a float");
    *out = (float)d;
    return JK_OK;
}

extern "C" jk_status jk_gguf_bool(const jk_gguf* g, const char* key, int64_t index, int* out) {
    const Value* v;
    if (jk_status st = value_at(g, key, index, &v)) return st;
    if (!out || v->kind != K_BOOL) return fail(JK_ERR_INVALID, std::string("Invalid GGUF file: ") + key + " is not a boolean");
    *out = (int)v->u;
    return JK_OK;
}

extern "C" jk_status jk_gguf_str(const jk_gguf* g, const char* key, int64_t index, const char** out, size_t* len) {
    const Value* v;
    if (jk_status st = value_at(g, key, index, &v)) return st;
    if (!out || v->kind != K_STRING) return fail(JK_ERR_INVALID, std::string("Invalid GGUF file: ") + key + " is not a string");
    *out = v->s.c_str();
    if (len) *len = v->s.size();
    return JK_OK;
}

extern "C" jk_status jk_qmatrix_from_gguf(int device, const jk_gguf* g, const char* name, jk_qmatrix** out) {
    if (!g || !out) return fail(JK_ERR_INVALID, "null pointer");
    const Tensor* t = find_tensor(g, name);
    if (!t) return missing_tensor(name);
    if (!t->known) return fail(JK_ERR_INVALID, "Invalid GGUF file: tensor " + t->name + " has unsupported type " + type_debug(t->type));
    const uint64_t k = t->dims[0];
    const uint64_t n = t->dims.size() > 1 ? t->dims[1] : 1;
    uint64_t experts = 1;
    for (size_t d = 2; d < t->dims.size(); ++d) experts *= t->dims[d];
    std::vector<uint8_t> raw;
    try {
        raw.resize((size_t)t->bytes);
    } catch (const std::bad_alloc&) {
        return fail(JK_ERR_INVALID, "qmatrix_from_gguf: host memory for tensor " + t->name);
    }
    if (jk_status st = jk_gguf_read(g, name, 0, t->bytes, raw.data())) return st;
    return jk_qmatrix_upload(device, t->type, (size_t)n, (size_t)k, (size_t)experts, raw.data(), raw.size(), out);
}
