// hd_gguf.cu -- GGUF v2/v3 reader (host code): header, metadata, tensor index
// and tensor bytes of a GGUF file, and upload of its quantized matrices as
// device weight handles.
//
// Replaces GgufLoader::load_std / GgufTensorIndex::parse / tensor_bytes
// (src/x/loader/gguf/loader.rs:64-141, tensor_index.rs:24-170,
// header.rs:54-84), which read value types as one byte, skip arrays by a
// guessed element size, read tensor infos in the wrong field order (type
// before dims), ignore the data-section alignment and size tensors by a fixed
// bytes-per-element.  This reader follows the published GGUF layout (as
// written by gguf-py 0.19.0, GGUFWriter):
//   u32 magic "GGUF", u32 version (2 or 3), u64 tensor_count, u64 kv_count;
//   kv_count x { string key, u32 value_type, value };
//   tensor_count x { string name, u32 n_dims, u64 dims[n_dims] (dims[0] is the
//     contiguous one), u32 ggml_type, u64 offset };
//   padding to general.alignment (default 32); tensor data, each tensor at
//   data_start + offset.
// Strings are u64 length + bytes (no NUL); arrays are u32 element type, u64
// count, elements.  Every read is bounds-checked: a malformed or truncated
// file is an error (HD_E_ARG with a message), never an out-of-range read.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "hd_internal.cuh"

namespace {

enum : uint32_t {
    V_U8 = 0, V_I8 = 1, V_U16 = 2, V_I16 = 3, V_U32 = 4, V_I32 = 5, V_F32 = 6, V_BOOL = 7,
    V_STR = 8, V_ARR = 9, V_U64 = 10, V_I64 = 11, V_F64 = 12
};

// Bytes of a scalar value type (0 for string/array/unknown).
int scalar_size(uint32_t t) {
    switch (t) {
    case V_U8: case V_I8: case V_BOOL: return 1;
    case V_U16: case V_I16: return 2;
    case V_U32: case V_I32: case V_F32: return 4;
    case V_U64: case V_I64: case V_F64: return 8;
    default: return 0;
    }
}

// ggml block size and bytes per block of the types whose size this reader
// knows (ggml-common.h block structs; gguf-py GGML_QUANT_SIZES).  0 = unknown.
void type_block(int t, int64_t &blck, int64_t &bytes) {
    static const int64_t tab[][3] = {
        {0, 1, 4},     {1, 1, 2},     {2, 32, 18},   {3, 32, 20},   {6, 32, 22},   {7, 32, 24},
        {8, 32, 34},   {9, 32, 36},   {10, 256, 84}, {11, 256, 110}, {12, 256, 144}, {13, 256, 176},
        {14, 256, 210}, {15, 256, 292}, {24, 1, 1},   {25, 1, 2},    {26, 1, 4},    {27, 1, 8},
        {28, 1, 8},    {30, 1, 2}};
    blck = 0;
    bytes = 0;
    for (const auto &r : tab)
        if (r[0] == t) {
            blck = r[1];
            bytes = r[2];
        }
}

thread_local std::string g_err;

int gfail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

}  // namespace

struct hd_gguf {
    std::vector<uint8_t> owned;   // bytes of hd_gguf_open_memory
    void *map = nullptr;          // mmap of hd_gguf_open
    size_t map_len = 0;
    const uint8_t *p = nullptr;   // file bytes
    uint64_t n = 0;
    uint32_t version = 0;
    uint64_t alignment = 32, data_start = 0;
    struct KV {
        std::string key;
        uint32_t type = 0, arr_type = 0;
        uint64_t off = 0;               // offset of the value (scalars, strings) or first element (arrays)
        uint64_t arr_n = 0;
        std::vector<uint64_t> str_off;  // string arrays: offset of each element's length field
    };
    struct TI {
        std::string name;
        int32_t n_dims = 0, type = 0;
        int64_t dims[4] = {1, 1, 1, 1};
        uint64_t rel = 0, nbytes = 0;
    };
    std::vector<KV> kv;
    std::vector<TI> ti;
    ~hd_gguf() {
        if (map) munmap(map, map_len);
    }
};

namespace {

struct Cur {
    const uint8_t *p;
    uint64_t n, o = 0;
    bool take(uint64_t k) {
        if (k > n - o) return false;
        o += k;
        return true;
    }
    template <class T>
    bool get(T &v) {
        if (sizeof(T) > n - o) return false;
        memcpy(&v, p + o, sizeof(T));
        o += sizeof(T);
        return true;
    }
    bool str(std::string &s) {
        uint64_t len;
        if (!get(len) || len > n - o) return false;
        s.assign((const char *)p + o, (size_t)len);
        o += len;
        return true;
    }
};

int parse(hd_gguf *g) {
    Cur c{g->p, g->n};
    uint32_t magic;
    if (!c.get(magic) || memcmp(g->p, "GGUF", 4) != 0) return gfail(HD_E_ARG, "gguf: bad magic (not a GGUF file)");
    if (!c.get(g->version)) return gfail(HD_E_ARG, "gguf: truncated header");
    if (g->version != 2 && g->version != 3)
        return gfail(HD_E_UNSUPPORTED, "gguf: version %u (2 and 3 are read; a byte-swapped version is a big-endian file)",
                     g->version);
    uint64_t nt, nk;
    if (!c.get(nt) || !c.get(nk)) return gfail(HD_E_ARG, "gguf: truncated header");
    // every kv takes at least 8 + 4 + 1 bytes, every tensor info 8 + 4 + 4 + 8
    if (nk > g->n / 13 || nt > g->n / 24) return gfail(HD_E_ARG, "gguf: counts (%llu kv, %llu tensors) exceed the file",
                                                      (unsigned long long)nk, (unsigned long long)nt);
    g->kv.resize(nk);
    for (uint64_t i = 0; i < nk; i++) {
        hd_gguf::KV &k = g->kv[i];
        if (!c.str(k.key) || !c.get(k.type)) return gfail(HD_E_ARG, "gguf: truncated metadata key %llu", (unsigned long long)i);
        k.off = c.o;
        if (k.type == V_STR) {
            std::string s;
            if (!c.str(s)) return gfail(HD_E_ARG, "gguf: truncated string value of '%s'", k.key.c_str());
        } else if (k.type == V_ARR) {
            if (!c.get(k.arr_type) || !c.get(k.arr_n)) return gfail(HD_E_ARG, "gguf: truncated array of '%s'", k.key.c_str());
            k.off = c.o;
            if (k.arr_type == V_STR) {
                if (k.arr_n > (c.n - c.o) / 8) return gfail(HD_E_ARG, "gguf: array '%s' exceeds the file", k.key.c_str());
                k.str_off.resize(k.arr_n);
                for (uint64_t j = 0; j < k.arr_n; j++) {
                    k.str_off[j] = c.o;
                    std::string s;
                    if (!c.str(s)) return gfail(HD_E_ARG, "gguf: truncated string %llu of '%s'", (unsigned long long)j, k.key.c_str());
                }
            } else {
                const int es = scalar_size(k.arr_type);
                if (es == 0) return gfail(HD_E_UNSUPPORTED, "gguf: array '%s' of element type %u", k.key.c_str(), k.arr_type);
                if (k.arr_n > (c.n - c.o) / es || !c.take(k.arr_n * es))
                    return gfail(HD_E_ARG, "gguf: array '%s' exceeds the file", k.key.c_str());
            }
        } else {
            const int es = scalar_size(k.type);
            if (es == 0) return gfail(HD_E_ARG, "gguf: value type %u of '%s'", k.type, k.key.c_str());
            if (!c.take(es)) return gfail(HD_E_ARG, "gguf: truncated value of '%s'", k.key.c_str());
        }
        if (k.key == "general.alignment") {
            uint32_t a = 0;
            if (k.type != V_U32) return gfail(HD_E_ARG, "gguf: general.alignment has type %u (u32 expected)", k.type);
            memcpy(&a, g->p + k.off, 4);
            if (a == 0 || (a & (a - 1)) != 0) return gfail(HD_E_ARG, "gguf: general.alignment %u is not a power of two", a);
            g->alignment = a;
        }
    }
    g->ti.resize(nt);
    for (uint64_t i = 0; i < nt; i++) {
        hd_gguf::TI &t = g->ti[i];
        uint32_t nd, ty;
        if (!c.str(t.name) || !c.get(nd)) return gfail(HD_E_ARG, "gguf: truncated tensor info %llu", (unsigned long long)i);
        if (nd < 1 || nd > 4) return gfail(HD_E_ARG, "gguf: tensor '%s' has %u dims (1..4)", t.name.c_str(), nd);
        t.n_dims = (int32_t)nd;
        for (uint32_t d = 0; d < nd; d++) {
            uint64_t v;
            if (!c.get(v)) return gfail(HD_E_ARG, "gguf: truncated dims of '%s'", t.name.c_str());
            if (v == 0 || v > ((uint64_t)1 << 40)) return gfail(HD_E_ARG, "gguf: tensor '%s' dim %u = %llu", t.name.c_str(), d, (unsigned long long)v);
            t.dims[d] = (int64_t)v;
        }
        if (!c.get(ty) || !c.get(t.rel)) return gfail(HD_E_ARG, "gguf: truncated tensor info of '%s'", t.name.c_str());
        t.type = (int32_t)ty;
        int64_t blck, bb;
        type_block(t.type, blck, bb);
        if (blck > 0) {
            if (t.dims[0] % blck != 0)
                return gfail(HD_E_ARG, "gguf: tensor '%s': %lld columns is not a multiple of the type's block %lld",
                             t.name.c_str(), (long long)t.dims[0], (long long)blck);
            const double nb = (double)(t.dims[0] / blck) * bb * t.dims[1] * t.dims[2] * t.dims[3];
            if (nb > (double)g->n) return gfail(HD_E_ARG, "gguf: tensor '%s' is larger than the file", t.name.c_str());
            t.nbytes = (uint64_t)(t.dims[0] / blck) * bb * t.dims[1] * t.dims[2] * t.dims[3];
        }
    }
    g->data_start = (c.o + g->alignment - 1) / g->alignment * g->alignment;
    if (nt > 0 && g->data_start > g->n) return gfail(HD_E_ARG, "gguf: no data section");
    for (const hd_gguf::TI &t : g->ti) {
        if (t.rel % g->alignment != 0)
            return gfail(HD_E_ARG, "gguf: tensor '%s' offset %llu is not a multiple of the alignment %llu",
                         t.name.c_str(), (unsigned long long)t.rel, (unsigned long long)g->alignment);
        if (t.rel > g->n - g->data_start || t.nbytes > g->n - g->data_start - t.rel)
            return gfail(HD_E_ARG, "gguf: data of tensor '%s' runs past the end of the file", t.name.c_str());
    }
    return HD_OK;
}

int finish_open(hd_gguf *g, hd_gguf **out) {
    const int rc = parse(g);
    if (rc) {
        delete g;
        return rc;
    }
    *out = g;
    return HD_OK;
}

bool kv_ok(const hd_gguf *g, int64_t i) { return g && i >= 0 && (uint64_t)i < g->kv.size(); }

}  // namespace

extern "C" {

const char *hd_gguf_error(void) { return g_err.c_str(); }

int hd_gguf_open(const char *path, hd_gguf **out) {
    if (!path || !out) return gfail(HD_E_ARG, "hd_gguf_open: null argument");
    *out = nullptr;
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return gfail(HD_E_ARG, "hd_gguf_open: cannot open '%s'", path);
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 24) {
        close(fd);
        return gfail(HD_E_ARG, "hd_gguf_open: '%s' is too small for a GGUF header", path);
    }
    void *m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (m == MAP_FAILED) return gfail(HD_E_ARG, "hd_gguf_open: cannot map '%s'", path);
    hd_gguf *g = new hd_gguf;
    g->map = m;
    g->map_len = (size_t)st.st_size;
    g->p = (const uint8_t *)m;
    g->n = (uint64_t)st.st_size;
    return finish_open(g, out);
}

int hd_gguf_open_memory(const uint8_t *bytes, size_t nbytes, hd_gguf **out) {
    if (!bytes || !out) return gfail(HD_E_ARG, "hd_gguf_open_memory: null argument");
    *out = nullptr;
    if (nbytes < 24) return gfail(HD_E_ARG, "hd_gguf_open_memory: %zu bytes is too small for a GGUF header", nbytes);
    hd_gguf *g = new hd_gguf;
    g->owned.assign(bytes, bytes + nbytes);
    g->p = g->owned.data();
    g->n = nbytes;
    return finish_open(g, out);
}

int hd_gguf_close(hd_gguf *g) {
    if (!g) return gfail(HD_E_ARG, "hd_gguf_close: null handle");
    delete g;
    return HD_OK;
}

int hd_gguf_counts(const hd_gguf *g, uint32_t *version, int64_t *n_tensors, int64_t *n_kv, uint64_t *alignment) {
    if (!g) return gfail(HD_E_ARG, "hd_gguf_counts: null handle");
    if (version) *version = g->version;
    if (n_tensors) *n_tensors = (int64_t)g->ti.size();
    if (n_kv) *n_kv = (int64_t)g->kv.size();
    if (alignment) *alignment = g->alignment;
    return HD_OK;
}

int hd_gguf_tensor(const hd_gguf *g, int64_t i, hd_gguf_tensor_info *out) {
    if (!g || !out) return gfail(HD_E_ARG, "hd_gguf_tensor: null argument");
    if (i < 0 || (uint64_t)i >= g->ti.size()) return gfail(HD_E_ARG, "hd_gguf_tensor: index %lld out of range", (long long)i);
    const hd_gguf::TI &t = g->ti[(size_t)i];
    out->name = t.name.c_str();
    out->ggml_type = t.type;
    out->n_dims = t.n_dims;
    for (int d = 0; d < 4; d++) out->dims[d] = t.dims[d];
    out->offset = g->data_start + t.rel;
    out->nbytes = t.nbytes;
    out->data = g->p + g->data_start + t.rel;
    return HD_OK;
}

int hd_gguf_find_tensor(const hd_gguf *g, const char *name, int64_t *index) {
    if (!g || !name || !index) return gfail(HD_E_ARG, "hd_gguf_find_tensor: null argument");
    for (size_t i = 0; i < g->ti.size(); i++)
        if (g->ti[i].name == name) {
            *index = (int64_t)i;
            return HD_OK;
        }
    *index = -1;
    return gfail(HD_E_ARG, "hd_gguf_find_tensor: no tensor named '%s'", name);
}

int hd_gguf_kv(const hd_gguf *g, int64_t i, const char **key, int32_t *type, int32_t *arr_type, uint64_t *arr_len) {
    if (!kv_ok(g, i)) return gfail(HD_E_ARG, "hd_gguf_kv: bad handle or index");
    const hd_gguf::KV &k = g->kv[(size_t)i];
    if (key) *key = k.key.c_str();
    if (type) *type = (int32_t)k.type;
    if (arr_type) *arr_type = k.type == V_ARR ? (int32_t)k.arr_type : -1;
    if (arr_len) *arr_len = k.type == V_ARR ? k.arr_n : 0;
    return HD_OK;
}

int hd_gguf_find_key(const hd_gguf *g, const char *key, int64_t *index) {
    if (!g || !key || !index) return gfail(HD_E_ARG, "hd_gguf_find_key: null argument");
    for (size_t i = 0; i < g->kv.size(); i++)
        if (g->kv[i].key == key) {
            *index = (int64_t)i;
            return HD_OK;
        }
    *index = -1;
    return gfail(HD_E_ARG, "hd_gguf_find_key: no key '%s'", key);
}

int hd_gguf_kv_int(const hd_gguf *g, int64_t i, int64_t *out) {
    if (!kv_ok(g, i) || !out) return gfail(HD_E_ARG, "hd_gguf_kv_int: bad argument");
    const hd_gguf::KV &k = g->kv[(size_t)i];
    const uint8_t *v = g->p + k.off;
    switch (k.type) {
    case V_U8: *out = *v; break;
    case V_I8: *out = (int8_t)*v; break;
    case V_BOOL: *out = *v != 0; break;
    case V_U16: { uint16_t x; memcpy(&x, v, 2); *out = x; break; }
    case V_I16: { int16_t x; memcpy(&x, v, 2); *out = x; break; }
    case V_U32: { uint32_t x; memcpy(&x, v, 4); *out = x; break; }
    case V_I32: { int32_t x; memcpy(&x, v, 4); *out = x; break; }
    case V_I64: { int64_t x; memcpy(&x, v, 8); *out = x; break; }
    case V_U64: {
        uint64_t x;
        memcpy(&x, v, 8);
        if (x > (uint64_t)INT64_MAX) return gfail(HD_E_ARG, "hd_gguf_kv_int: '%s' does not fit in int64", k.key.c_str());
        *out = (int64_t)x;
        break;
    }
    default: return gfail(HD_E_TYPE, "hd_gguf_kv_int: '%s' has value type %u", k.key.c_str(), k.type);
    }
    return HD_OK;
}

int hd_gguf_kv_float(const hd_gguf *g, int64_t i, double *out) {
    if (!kv_ok(g, i) || !out) return gfail(HD_E_ARG, "hd_gguf_kv_float: bad argument");
    const hd_gguf::KV &k = g->kv[(size_t)i];
    if (k.type == V_F32) {
        float x;
        memcpy(&x, g->p + k.off, 4);
        *out = x;
        return HD_OK;
    }
    if (k.type == V_F64) {
        memcpy(out, g->p + k.off, 8);
        return HD_OK;
    }
    int64_t v;
    const int rc = hd_gguf_kv_int(g, i, &v);
    if (rc) return gfail(HD_E_TYPE, "hd_gguf_kv_float: '%s' has value type %u", k.key.c_str(), k.type);
    *out = (double)v;
    return HD_OK;
}

int hd_gguf_kv_string(const hd_gguf *g, int64_t i, uint64_t j, const char **s, uint64_t *len) {
    if (!kv_ok(g, i) || !s || !len) return gfail(HD_E_ARG, "hd_gguf_kv_string: bad argument");
    const hd_gguf::KV &k = g->kv[(size_t)i];
    uint64_t at;
    if (k.type == V_STR && j == 0) at = k.off;
    else if (k.type == V_ARR && k.arr_type == V_STR && j < k.arr_n) at = k.str_off[j];
    else return gfail(HD_E_TYPE, "hd_gguf_kv_string: '%s' has no string %llu", k.key.c_str(), (unsigned long long)j);
    memcpy(len, g->p + at, 8);
    *s = (const char *)g->p + at + 8;
    return HD_OK;
}

int hd_gguf_kv_array(const hd_gguf *g, int64_t i, const void **data, uint64_t *n) {
    if (!kv_ok(g, i) || !data || !n) return gfail(HD_E_ARG, "hd_gguf_kv_array: bad argument");
    const hd_gguf::KV &k = g->kv[(size_t)i];
    if (k.type != V_ARR && scalar_size(k.type) > 0) {  // a numeric scalar: an array of one
        *data = g->p + k.off;
        *n = 1;
        return HD_OK;
    }
    if (k.type != V_ARR || k.arr_type == V_STR)
        return gfail(HD_E_TYPE, "hd_gguf_kv_array: '%s' is not numeric", k.key.c_str());
    *data = g->p + k.off;
    *n = k.arr_n;
    return HD_OK;
}

int hd_gguf_upload(hd_ctx *ctx, const hd_gguf *g, const char *name, hd_weight **out) {
    if (!ctx || !g || !name || !out) return hd_fail(ctx, HD_E_ARG, "hd_gguf_upload: null argument");
    int64_t i;
    if (hd_gguf_find_tensor(g, name, &i)) return hd_fail(ctx, HD_E_ARG, "%s", g_err.c_str());
    const hd_gguf::TI &t = g->ti[(size_t)i];
    if (t.type != HD_TYPE_Q8_0 && t.type != HD_TYPE_Q5_0 && t.type != HD_TYPE_Q4_K && t.type != HD_TYPE_Q6_K)
        return hd_fail(ctx, HD_E_TYPE, "hd_gguf_upload: tensor '%s' has ggml type %d (Q8_0, Q5_0, Q4_K, Q6_K upload)",
                       name, t.type);
    if (t.n_dims > 2 && (t.dims[2] != 1 || t.dims[3] != 1))
        return hd_fail(ctx, HD_E_SHAPE, "hd_gguf_upload: tensor '%s' is not a matrix", name);
    // GGUF dims[0] is the contiguous axis: a [rows x cols] weight is dims {cols, rows}
    return hd_weight_upload(ctx, g->p + g->data_start + t.rel, (size_t)t.nbytes, t.type, t.dims[1], t.dims[0], out);
}

}  // extern "C"
