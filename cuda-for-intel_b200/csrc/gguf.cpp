// gguf.cpp -- read-only GGUF v2/v3 parser (include/cfi_gguf.h).
//
// Layout (the published GGUF specification): "GGUF", u32 version, u64 tensor count, u64
// metadata count; metadata entries (string key, u32 value type, value; strings are u64 length +
// bytes, arrays u32 element type + u64 count + elements); tensor infos (string name, u32 n_dims,
// u64 ne[n_dims], u32 ggml type, u64 offset from the data section); the data section starts at the
// next multiple of general.alignment (default 32) after the infos.  All integers little-endian.
#include <fcntl.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <string>
#include <vector>

#include "../../include/cfi_gguf.h"

namespace {

struct Kv {
    std::string key;
    int type = 0, elem_type = 0;
    uint64_t count = 0;  // array length
    uint64_t off = 0;    // file offset of the value (arrays: of the first element)
};

struct Tensor {
    std::string name;
    uint32_t type = 0, n_dims = 0;
    uint64_t dims[4] = {1, 1, 1, 1};
    uint64_t offset = 0, nbytes = 0;
};

// ggml block sizes: (values per block, bytes per block); ggml.h type ids
bool type_block(uint32_t t, uint64_t* qk, uint64_t* bytes) {
    static const struct {
        uint32_t t;
        uint64_t qk, b;
    } tab[] = {{0, 1, 4},      {1, 1, 2},      {2, 32, 18},    {3, 32, 20},    {6, 32, 22},   {7, 32, 24},
               {8, 32, 34},    {9, 32, 36},    {10, 256, 84},  {11, 256, 110}, {12, 256, 144}, {13, 256, 176},
               {14, 256, 210}, {15, 256, 292}, {24, 1, 1},     {25, 1, 2},     {26, 1, 4},     {27, 1, 8},
               {28, 1, 8},     {30, 1, 2}};
    for (const auto& e : tab)
        if (e.t == t) {
            *qk = e.qk;
            *bytes = e.b;
            return true;
        }
    return false;
}

size_t scalar_size(int t) {
    switch (t) {
    case CFI_GGUF_U8: case CFI_GGUF_I8: case CFI_GGUF_BOOL: return 1;
    case CFI_GGUF_U16: case CFI_GGUF_I16: return 2;
    case CFI_GGUF_U32: case CFI_GGUF_I32: case CFI_GGUF_F32: return 4;
    case CFI_GGUF_U64: case CFI_GGUF_I64: case CFI_GGUF_F64: return 8;
    default: return 0;
    }
}

}  // namespace

struct cfi_gguf {
    int fd = -1;
    const uint8_t* map = nullptr;
    uint64_t size = 0;
    uint32_t version = 0;
    uint64_t alignment = 32, data_off = 0;
    std::vector<Kv> kvs;
    std::vector<Tensor> tensors;
};

namespace {

struct Reader {
    const uint8_t* p;
    uint64_t size, pos = 0;
    bool ok = true;
    bool need(uint64_t n) {
        if (!ok || n > size || pos > size - n) ok = false;
        return ok;
    }
    template <class T> T get() {
        T v{};
        if (need(sizeof(T))) {
            memcpy(&v, p + pos, sizeof(T));
            pos += sizeof(T);
        }
        return v;
    }
    bool str(std::string* out) {
        const uint64_t n = get<uint64_t>();
        if (!need(n)) return false;
        if (out) out->assign(reinterpret_cast<const char*>(p + pos), n);
        pos += n;
        return true;
    }
    // skips one value of type t (strings and nested arrays included), depth-limited
    bool skip(int t, int depth = 0) {
        if (depth > 4) return ok = false;
        if (t == CFI_GGUF_STRING) return str(nullptr);
        if (t == CFI_GGUF_ARRAY) {
            const int et = (int)get<uint32_t>();
            const uint64_t n = get<uint64_t>();
            if (!ok) return false;
            const size_t es = scalar_size(et);
            if (es) {
                if (n > size / es || !need(n * es)) return ok = false;
                pos += n * es;
                return true;
            }
            for (uint64_t i = 0; i < n && ok; i++) skip(et, depth + 1);
            return ok;
        }
        const size_t s = scalar_size(t);
        if (!s || !need(s)) return ok = false;
        pos += s;
        return true;
    }
};

int fail(char* why, size_t len, const std::string& m) {
    if (why && len) snprintf(why, len, "%s", m.c_str());
    return -1;
}

}  // namespace

extern "C" int cfi_gguf_open(const char* path, cfi_gguf** out, char* why, size_t why_len) {
    if (!path || !out) return fail(why, why_len, "null argument");
    *out = nullptr;
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return fail(why, why_len, std::string("cannot open ") + path);
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 24) {
        close(fd);
        return fail(why, why_len, "not a GGUF file (too short)");
    }
    void* m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (m == MAP_FAILED) {
        close(fd);
        return fail(why, why_len, "mmap failed");
    }
    cfi_gguf* f = new cfi_gguf;
    f->fd = fd;
    f->map = static_cast<const uint8_t*>(m);
    f->size = (uint64_t)st.st_size;
    auto bad = [&](const std::string& msg) {
        cfi_gguf_close(f);
        return fail(why, why_len, msg);
    };
    Reader r{f->map, f->size};
    if (r.get<uint32_t>() != 0x46554747u) return bad("bad magic (not GGUF)");
    f->version = r.get<uint32_t>();
    if (f->version != 2 && f->version != 3) return bad("unsupported GGUF version " + std::to_string(f->version));
    const uint64_t nt = r.get<uint64_t>(), nkv = r.get<uint64_t>();
    if (nt > f->size / 24 || nkv > f->size / 12) return bad("tensor or metadata count larger than the file");
    f->kvs.reserve((size_t)nkv);
    for (uint64_t i = 0; i < nkv && r.ok; i++) {
        Kv kv;
        if (!r.str(&kv.key)) break;
        kv.type = (int)r.get<uint32_t>();
        if (!r.ok) break;
        if (kv.type == CFI_GGUF_ARRAY) {
            kv.elem_type = (int)r.get<uint32_t>();
            kv.count = r.get<uint64_t>();
            kv.off = r.pos;
            // rewind to the array header and skip it whole
            r.pos -= 12;
            if (!r.skip(CFI_GGUF_ARRAY)) break;
        } else {
            kv.off = r.pos;
            if (!r.skip(kv.type)) break;
        }
        f->kvs.push_back(kv);
    }
    if (!r.ok) return bad("truncated or malformed metadata");
    const int64_t ai = cfi_gguf_find_key(f, "general.alignment");
    if (ai >= 0) {
        int64_t a = 0;
        if (cfi_gguf_get_i64(f, ai, 0, &a) != 0 || a <= 0 || (a & (a - 1))) return bad("general.alignment is not a power of two");
        f->alignment = (uint64_t)a;
    }
    f->tensors.reserve((size_t)nt);
    for (uint64_t i = 0; i < nt && r.ok; i++) {
        Tensor t;
        if (!r.str(&t.name)) break;
        t.n_dims = r.get<uint32_t>();
        if (!r.ok || t.n_dims == 0 || t.n_dims > 4) return bad("tensor " + t.name + ": bad dimension count");
        uint64_t n = 1;
        for (uint32_t d = 0; d < t.n_dims; d++) {
            t.dims[d] = r.get<uint64_t>();
            if (t.dims[d] && n > UINT64_MAX / t.dims[d]) return bad("tensor " + t.name + ": size overflows");
            n *= t.dims[d];
        }
        t.type = r.get<uint32_t>();
        t.offset = r.get<uint64_t>();
        t.nbytes = cfi_gguf_type_bytes(t.type, n);
        uint64_t qk = 0, bb = 0;
        if (type_block(t.type, &qk, &bb) && t.dims[0] % qk) return bad("tensor " + t.name + ": rows are not whole blocks");
        f->tensors.push_back(t);
    }
    if (!r.ok) return bad("truncated tensor table");
    f->data_off = (r.pos + f->alignment - 1) / f->alignment * f->alignment;
    for (const auto& t : f->tensors) {
        if (t.offset % f->alignment) return bad("tensor " + t.name + ": data offset not aligned");
        if (f->data_off > f->size || t.offset > f->size - f->data_off || t.nbytes > f->size - f->data_off - t.offset)
            return bad("tensor " + t.name + ": data past the end of the file");
    }
    *out = f;
    return 0;
}

extern "C" void cfi_gguf_close(cfi_gguf* f) {
    if (!f) return;
    if (f->map) munmap(const_cast<uint8_t*>(f->map), (size_t)f->size);
    if (f->fd >= 0) close(f->fd);
    delete f;
}

extern "C" uint32_t cfi_gguf_version(const cfi_gguf* f) { return f ? f->version : 0; }
extern "C" uint64_t cfi_gguf_alignment(const cfi_gguf* f) { return f ? f->alignment : 0; }
extern "C" uint64_t cfi_gguf_data_offset(const cfi_gguf* f) { return f ? f->data_off : 0; }
extern "C" int64_t cfi_gguf_kv_count(const cfi_gguf* f) { return f ? (int64_t)f->kvs.size() : -1; }

extern "C" int64_t cfi_gguf_find_key(const cfi_gguf* f, const char* key) {
    if (!f || !key) return -1;
    for (size_t i = 0; i < f->kvs.size(); i++)
        if (f->kvs[i].key == key) return (int64_t)i;
    return -1;
}

extern "C" const char* cfi_gguf_key(const cfi_gguf* f, int64_t i) {
    return f && i >= 0 && (size_t)i < f->kvs.size() ? f->kvs[(size_t)i].key.c_str() : nullptr;
}

extern "C" int cfi_gguf_kv_type(const cfi_gguf* f, int64_t i, int* elem_type, uint64_t* count) {
    if (!f || i < 0 || (size_t)i >= f->kvs.size()) return -1;
    const Kv& kv = f->kvs[(size_t)i];
    if (elem_type) *elem_type = kv.elem_type;
    if (count) *count = kv.type == CFI_GGUF_ARRAY ? kv.count : 1;
    return kv.type;
}

namespace {
// file offset and type of scalar element j of entry i (the value itself, or array element j)
bool element(const cfi_gguf* f, int64_t i, uint64_t j, uint64_t* off, int* type) {
    if (!f || i < 0 || (size_t)i >= f->kvs.size()) return false;
    const Kv& kv = f->kvs[(size_t)i];
    if (kv.type != CFI_GGUF_ARRAY) {
        if (j != 0) return false;
        *off = kv.off;
        *type = kv.type;
        return true;
    }
    if (j >= kv.count) return false;
    const size_t es = scalar_size(kv.elem_type);
    if (es) {
        *off = kv.off + j * es;
        *type = kv.elem_type;
        return true;
    }
    if (kv.elem_type != CFI_GGUF_STRING) return false;
    Reader r{f->map, f->size, kv.off};
    for (uint64_t k = 0; k < j && r.ok; k++) r.str(nullptr);
    if (!r.ok) return false;
    *off = r.pos;
    *type = CFI_GGUF_STRING;
    return true;
}
}  // namespace

extern "C" int cfi_gguf_get_i64(const cfi_gguf* f, int64_t i, uint64_t j, int64_t* out) {
    uint64_t off = 0;
    int t = 0;
    if (!out || !element(f, i, j, &off, &t)) return -1;
    const uint8_t* p = f->map + off;
    switch (t) {
    case CFI_GGUF_U8: case CFI_GGUF_BOOL: *out = *p; return 0;
    case CFI_GGUF_I8: *out = (int8_t)*p; return 0;
    case CFI_GGUF_U16: { uint16_t v; memcpy(&v, p, 2); *out = v; return 0; }
    case CFI_GGUF_I16: { int16_t v; memcpy(&v, p, 2); *out = v; return 0; }
    case CFI_GGUF_U32: { uint32_t v; memcpy(&v, p, 4); *out = v; return 0; }
    case CFI_GGUF_I32: { int32_t v; memcpy(&v, p, 4); *out = v; return 0; }
    case CFI_GGUF_U64: { uint64_t v; memcpy(&v, p, 8); if (v > (uint64_t)INT64_MAX) return -1; *out = (int64_t)v; return 0; }
    case CFI_GGUF_I64: { int64_t v; memcpy(&v, p, 8); *out = v; return 0; }
    default: return -1;
    }
}

extern "C" int cfi_gguf_get_f64(const cfi_gguf* f, int64_t i, uint64_t j, double* out) {
    uint64_t off = 0;
    int t = 0;
    if (!out || !element(f, i, j, &off, &t)) return -1;
    const uint8_t* p = f->map + off;
    if (t == CFI_GGUF_F32) {
        float v;
        memcpy(&v, p, 4);
        *out = v;
        return 0;
    }
    if (t == CFI_GGUF_F64) {
        memcpy(out, p, 8);
        return 0;
    }
    int64_t v = 0;
    if (cfi_gguf_get_i64(f, i, j, &v) != 0) return -1;
    *out = (double)v;
    return 0;
}

extern "C" int cfi_gguf_get_str(const cfi_gguf* f, int64_t i, uint64_t j, const char** s, uint64_t* len) {
    uint64_t off = 0;
    int t = 0;
    if (!s || !len || !element(f, i, j, &off, &t) || t != CFI_GGUF_STRING) return -1;
    uint64_t n;
    memcpy(&n, f->map + off, 8);
    *s = reinterpret_cast<const char*>(f->map + off + 8);
    *len = n;
    return 0;
}

extern "C" int64_t cfi_gguf_tensor_count(const cfi_gguf* f) { return f ? (int64_t)f->tensors.size() : -1; }

extern "C" int64_t cfi_gguf_find_tensor(const cfi_gguf* f, const char* name) {
    if (!f || !name) return -1;
    for (size_t i = 0; i < f->tensors.size(); i++)
        if (f->tensors[i].name == name) return (int64_t)i;
    return -1;
}

extern "C" int cfi_gguf_tensor_info(const cfi_gguf* f, int64_t i, const char** name, uint32_t* ggml_type,
                                    uint32_t* n_dims, uint64_t dims[4], uint64_t* nbytes, const void** data) {
    if (!f || i < 0 || (size_t)i >= f->tensors.size()) return -1;
    const Tensor& t = f->tensors[(size_t)i];
    if (name) *name = t.name.c_str();
    if (ggml_type) *ggml_type = t.type;
    if (n_dims) *n_dims = t.n_dims;
    if (dims)
        for (int d = 0; d < 4; d++) dims[d] = t.dims[d];
    if (nbytes) *nbytes = t.nbytes;
    if (data) *data = f->map + f->data_off + t.offset;
    return 0;
}

extern "C" uint64_t cfi_gguf_type_bytes(uint32_t ggml_type, uint64_t n) {
    uint64_t qk = 0, bb = 0;
    if (!type_block(ggml_type, &qk, &bb) || n % qk) return 0;
    return n / qk * bb;
}
