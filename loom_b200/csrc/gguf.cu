// gguf.cu -- host-side GGUF v2/v3 reader: header, metadata, tensor table and
// the checked tensor resolve the engine does before any byte reaches the
// device. Pure host code (no CUDA calls); it lives in the backend library so
// a C/Zig caller gets the tensor table and the upload from one .so.
//
// Behaviour follows src/gguf/gguf.zig:251-325 (parse), :157-210 (metadata
// values, array nesting cap), :82-126 (the Parsed getters) and
// src/gguf/llama.zig:259-273 with src/gguf/ggml.zig:143-153 (resolve with
// overflow-checked sizes). The error names are the reference's error set.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <string>
#include <vector>

#include "../../include/loom_cuda.h"

namespace {

thread_local std::string g_gguf_err;

enum VType : uint32_t {
    V_U8 = 0, V_I8 = 1, V_U16 = 2, V_I16 = 3, V_U32 = 4, V_I32 = 5, V_F32 = 6, V_BOOL = 7,
    V_STR = 8, V_ARR = 9, V_U64 = 10, V_I64 = 11, V_F64 = 12
};

struct Meta {
    const char *key;
    size_t key_len;
    int kind;  // LOOM_GGUF_META_*
    int64_t i = 0;
    uint64_t u = 0;
    double f = 0;
    const char *s = nullptr;  // string value (view into the image)
    size_t s_len = 0;
    uint32_t elem_type = 0;   // arrays
    uint64_t count = 0;
    const uint8_t *arr = nullptr;  // first element of an f32 / i32 array, or the first string's length field
    uint64_t span_start = 0, span_end = 0;
};

struct Info {
    const char *name;
    size_t name_len;
    uint32_t n_dims;
    uint64_t dims[8];
    uint32_t type;
    uint64_t offset;
};

struct Err {
    const char *name;
};

struct Cursor {
    const uint8_t *buf;
    size_t len, pos = 0;
    const uint8_t *need(size_t n) {
        if (n > len - pos) throw Err{"TruncatedGguf"};
        const uint8_t *p = buf + pos;
        pos += n;
        return p;
    }
    uint32_t u32() {
        uint32_t v;
        std::memcpy(&v, need(4), 4);
        return v;
    }
    uint64_t u64() {
        uint64_t v;
        std::memcpy(&v, need(8), 8);
        return v;
    }
    const char *str(size_t *n) {
        const uint64_t l = u64();
        if (l > (1u << 24)) throw Err{"TruncatedGguf"};  // 16 MB string cap
        *n = (size_t)l;
        return reinterpret_cast<const char *>(need((size_t)l));
    }
};

constexpr uint32_t MAGIC = 0x46554747u;  // "GGUF" little-endian
constexpr int MAX_ARRAY_DEPTH = 4;
constexpr size_t HEAD_CAP = 64ull << 20;  // the parser reads at most 64 MB of header

void read_value(Cursor &c, uint32_t vt, int depth, Meta *m) {
    if (depth > MAX_ARRAY_DEPTH) throw Err{"ArrayNestingTooDeep"};
    Meta scratch{};
    Meta &o = m ? *m : scratch;
    switch (vt) {
        case V_U8: o.kind = LOOM_GGUF_META_UINT; o.u = *c.need(1); break;
        case V_I8: o.kind = LOOM_GGUF_META_INT; o.i = (int8_t)*c.need(1); break;
        case V_U16: { uint16_t v; std::memcpy(&v, c.need(2), 2); o.kind = LOOM_GGUF_META_UINT; o.u = v; break; }
        case V_I16: { int16_t v; std::memcpy(&v, c.need(2), 2); o.kind = LOOM_GGUF_META_INT; o.i = v; break; }
        case V_U32: o.kind = LOOM_GGUF_META_UINT; o.u = c.u32(); break;
        case V_I32: o.kind = LOOM_GGUF_META_INT; o.i = (int32_t)c.u32(); break;
        case V_F32: { uint32_t b = c.u32(); float f; std::memcpy(&f, &b, 4); o.kind = LOOM_GGUF_META_FLOAT; o.f = f; break; }
        case V_BOOL: o.kind = LOOM_GGUF_META_BOOL; o.u = *c.need(1) != 0; break;
        case V_STR: o.kind = LOOM_GGUF_META_STRING; o.s = c.str(&o.s_len); break;
        case V_U64: o.kind = LOOM_GGUF_META_UINT; o.u = c.u64(); break;
        case V_I64: o.kind = LOOM_GGUF_META_INT; o.i = (int64_t)c.u64(); break;
        case V_F64: { uint64_t b = c.u64(); double f; std::memcpy(&f, &b, 8); o.kind = LOOM_GGUF_META_FLOAT; o.f = f; break; }
        case V_ARR: {
            const uint32_t et = c.u32();
            const uint64_t count = c.u64();
            if (count > (1u << 24)) throw Err{"TruncatedGguf"};
            o.elem_type = et;
            o.count = count;
            o.arr = c.buf + c.pos;
            if (et == V_STR) {
                o.kind = LOOM_GGUF_META_ARRAY_STR;
                for (uint64_t k = 0; k < count; k++) {
                    size_t n;
                    c.str(&n);
                }
            } else if (et == V_F32 || et == V_I32) {
                o.kind = et == V_F32 ? LOOM_GGUF_META_ARRAY_F32 : LOOM_GGUF_META_ARRAY_I32;
                for (uint64_t k = 0; k < count; k++) c.need(4);
            } else {
                // other element types are skipped element by element (nested arrays recurse)
                o.kind = LOOM_GGUF_META_ARRAY;
                for (uint64_t k = 0; k < count; k++) read_value(c, et, depth + 1, nullptr);
            }
            break;
        }
        default: throw Err{"UnknownValueType"};
    }
}

bool add_ovf(uint64_t a, uint64_t b, uint64_t *r) { return __builtin_add_overflow(a, b, r); }
bool mul_ovf(uint64_t a, uint64_t b, uint64_t *r) { return __builtin_mul_overflow(a, b, r); }

// Block width in elements and bytes per block (src/gguf/ggml.zig:126-180,
// src/gguf/iq.zig:22-37). 0 bytes = not a supported type.
void type_geom(uint32_t t, uint64_t *elems, uint64_t *bytes) {
    *elems = 1;
    *bytes = 0;
    switch (t) {
        case 0: *bytes = 4; break;   // f32 (per element)
        case 1: *bytes = 2; break;   // f16
        case 2: *elems = 32; *bytes = 18; break;
        case 3: *elems = 32; *bytes = 20; break;
        case 6: *elems = 32; *bytes = 22; break;
        case 7: *elems = 32; *bytes = 24; break;
        case 8: *elems = 32; *bytes = 34; break;
        case 10: *elems = 256; *bytes = 84; break;
        case 11: *elems = 256; *bytes = 110; break;
        case 12: *elems = 256; *bytes = 144; break;
        case 13: *elems = 256; *bytes = 176; break;
        case 14: *elems = 256; *bytes = 210; break;
        case 16: *elems = 256; *bytes = 66; break;   // iq2_xxs
        case 17: *elems = 256; *bytes = 74; break;   // iq2_xs
        case 18: *elems = 256; *bytes = 98; break;   // iq3_xxs
        case 19: *elems = 256; *bytes = 50; break;   // iq1_s
        case 20: *elems = 32; *bytes = 18; break;    // iq4_nl
        case 21: *elems = 256; *bytes = 110; break;  // iq3_s
        case 22: *elems = 256; *bytes = 82; break;   // iq2_s
        case 23: *elems = 256; *bytes = 136; break;  // iq4_xs
        case 29: *elems = 256; *bytes = 56; break;   // iq1_m
        case 39: *elems = 32; *bytes = 17; break;    // mxfp4
        default: break;
    }
}

}  // namespace

struct loom_gguf {
    const uint8_t *image = nullptr;
    size_t size = 0;
    void *map = nullptr;  // set when loom_gguf_open mapped the file
    uint32_t version = 0;
    uint64_t alignment = 32, data_offset = 0;
    std::vector<Meta> meta;
    std::vector<Info> tensors;

    const Meta *find_meta(const char *key) const {
        const size_t n = std::strlen(key);
        for (const Meta &m : meta)
            if (m.key_len == n && std::memcmp(m.key, key, n) == 0) return &m;
        return nullptr;
    }
    const Info *find_tensor(const char *name) const {
        const size_t n = std::strlen(name);
        for (const Info &t : tensors)
            if (t.name_len == n && std::memcmp(t.name, name, n) == 0) return &t;
        return nullptr;
    }
};

namespace {

int parse_into(loom_gguf *g) {
    Cursor c{g->image, (size_t)std::min<uint64_t>(g->size, HEAD_CAP)};
    if (c.u32() != MAGIC) throw Err{"NotGguf"};
    g->version = c.u32();
    if (g->version < 2 || g->version > 3) throw Err{"UnsupportedGgufVersion"};
    const uint64_t tensor_count = c.u64();
    const uint64_t kv_count = c.u64();
    if (tensor_count > (1u << 20) || kv_count > (1u << 20)) throw Err{"TruncatedGguf"};
    g->meta.resize(kv_count);
    for (Meta &m : g->meta) {
        m.span_start = c.pos;
        m.key = c.str(&m.key_len);
        const uint32_t vt = c.u32();
        read_value(c, vt, 0, &m);
        m.span_end = c.pos;
    }
    g->tensors.resize(tensor_count);
    for (Info &t : g->tensors) {
        t.name = c.str(&t.name_len);
        t.n_dims = c.u32();
        // a 0-dim tensor or a 0-length dim leaves the element count meaningless
        if (t.n_dims == 0 || t.n_dims > 8) throw Err{"BadTensorDims"};
        uint64_t elems = 1;
        for (uint32_t d = 0; d < t.n_dims; d++) {
            t.dims[d] = c.u64();
            if (t.dims[d] == 0) throw Err{"BadTensorDims"};
            if (mul_ovf(elems, t.dims[d], &elems)) throw Err{"BadTensorDims"};
        }
        for (uint32_t d = t.n_dims; d < 8; d++) t.dims[d] = 1;
        t.type = c.u32();
        t.offset = c.u64();
    }
    uint64_t align = 32;
    if (const Meta *m = g->find_meta("general.alignment")) {
        if (m->kind == LOOM_GGUF_META_UINT) align = m->u;
        else if (m->kind == LOOM_GGUF_META_INT && m->i > 0) align = (uint64_t)m->i;
    }
    if (align == 0 || (align & (align - 1)) != 0) throw Err{"BadAlignment"};
    g->alignment = align;
    g->data_offset = (c.pos + align - 1) & ~(align - 1);
    if (g->data_offset > g->size) throw Err{"TruncatedGguf"};
    return 0;
}

loom_gguf *finish(loom_gguf *g) {
    try {
        parse_into(g);
    } catch (const Err &e) {
        g_gguf_err = e.name;
        loom_gguf_close(g);
        return nullptr;
    } catch (const std::bad_alloc &) {
        g_gguf_err = "OutOfMemory";
        loom_gguf_close(g);
        return nullptr;
    }
    g_gguf_err.clear();
    return g;
}

}  // namespace

extern "C" {

loom_gguf *loom_gguf_parse(const void *image, size_t bytes) {
    if (!image && bytes) {
        g_gguf_err = "NullImage";
        return nullptr;
    }
    loom_gguf *g = new loom_gguf;
    g->image = static_cast<const uint8_t *>(image);
    g->size = bytes;
    return finish(g);
}

loom_gguf *loom_gguf_open(const char *path) {
    const int fd = open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) {
        g_gguf_err = "FileNotFound";
        return nullptr;
    }
    struct stat st;
    if (fstat(fd, &st) != 0) {
        close(fd);
        g_gguf_err = "FileNotFound";
        return nullptr;
    }
    const size_t size = (size_t)st.st_size;
    void *map = size ? mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0) : nullptr;
    close(fd);
    if (size && map == MAP_FAILED) {
        g_gguf_err = "MapFailed";
        return nullptr;
    }
    loom_gguf *g = new loom_gguf;
    g->image = static_cast<const uint8_t *>(map);
    g->size = size;
    g->map = map;
    return finish(g);
}

const char *loom_gguf_error(void) { return g_gguf_err.empty() ? nullptr : g_gguf_err.c_str(); }

void loom_gguf_close(loom_gguf *g) {
    if (!g) return;
    if (g->map) munmap(g->map, g->size);
    delete g;
}

uint32_t loom_gguf_version(const loom_gguf *g) { return g->version; }
uint64_t loom_gguf_alignment(const loom_gguf *g) { return g->alignment; }
uint64_t loom_gguf_data_offset(const loom_gguf *g) { return g->data_offset; }
uint64_t loom_gguf_file_size(const loom_gguf *g) { return g->size; }
const void *loom_gguf_image(const loom_gguf *g) { return g->image; }
size_t loom_gguf_n_tensors(const loom_gguf *g) { return g->tensors.size(); }
size_t loom_gguf_n_meta(const loom_gguf *g) { return g->meta.size(); }

int loom_gguf_tensor_info(const loom_gguf *g, size_t i, loom_gguf_tensor *out) {
    if (i >= g->tensors.size()) return LOOM_CUDA_DECLINED;
    const Info &t = g->tensors[i];
    out->name = t.name;
    out->name_len = t.name_len;
    out->n_dims = t.n_dims;
    for (int d = 0; d < 8; d++) out->dims[d] = t.dims[d];
    out->ggml_type = t.type;
    out->offset = t.offset;
    return LOOM_CUDA_OK;
}

int loom_gguf_find_tensor(const loom_gguf *g, const char *name, loom_gguf_tensor *out) {
    const Info *t = g->find_tensor(name);
    if (!t) return LOOM_CUDA_DECLINED;
    return loom_gguf_tensor_info(g, (size_t)(t - g->tensors.data()), out);
}

int loom_gguf_meta(const loom_gguf *g, size_t i, loom_gguf_value *out) {
    if (i >= g->meta.size()) return LOOM_CUDA_DECLINED;
    const Meta &m = g->meta[i];
    out->key = m.key;
    out->key_len = m.key_len;
    out->kind = m.kind;
    out->i = m.i;
    out->u = m.u;
    out->f = m.f;
    out->str = m.s;
    out->str_len = m.s_len;
    out->elem_type = m.elem_type;
    out->count = m.count;
    out->array = m.arr;
    out->span_start = m.span_start;
    out->span_end = m.span_end;
    return LOOM_CUDA_OK;
}

int loom_gguf_find_meta(const loom_gguf *g, const char *key, loom_gguf_value *out) {
    const Meta *m = g->find_meta(key);
    if (!m) return LOOM_CUDA_DECLINED;
    return loom_gguf_meta(g, (size_t)(m - g->meta.data()), out);
}

int loom_gguf_get_uint(const loom_gguf *g, const char *key, uint64_t *out) {
    const Meta *m = g->find_meta(key);
    if (!m) return LOOM_CUDA_DECLINED;
    if (m->kind == LOOM_GGUF_META_UINT) *out = m->u;
    else if (m->kind == LOOM_GGUF_META_INT && m->i >= 0) *out = (uint64_t)m->i;
    else return LOOM_CUDA_DECLINED;
    return LOOM_CUDA_OK;
}

int loom_gguf_get_float(const loom_gguf *g, const char *key, double *out) {
    const Meta *m = g->find_meta(key);
    if (!m) return LOOM_CUDA_DECLINED;
    if (m->kind == LOOM_GGUF_META_FLOAT) *out = m->f;
    else if (m->kind == LOOM_GGUF_META_UINT) *out = (double)m->u;
    else if (m->kind == LOOM_GGUF_META_INT) *out = (double)m->i;
    else return LOOM_CUDA_DECLINED;
    return LOOM_CUDA_OK;
}

int loom_gguf_get_string(const loom_gguf *g, const char *key, const char **s, size_t *len) {
    const Meta *m = g->find_meta(key);
    if (!m || m->kind != LOOM_GGUF_META_STRING) return LOOM_CUDA_DECLINED;
    *s = m->s;
    *len = m->s_len;
    return LOOM_CUDA_OK;
}

int loom_gguf_get_bool(const loom_gguf *g, const char *key, int *out) {
    const Meta *m = g->find_meta(key);
    if (!m) return LOOM_CUDA_DECLINED;
    if (m->kind == LOOM_GGUF_META_BOOL || m->kind == LOOM_GGUF_META_UINT) *out = m->u != 0;
    else if (m->kind == LOOM_GGUF_META_INT) *out = m->i != 0;
    else return LOOM_CUDA_DECLINED;
    return LOOM_CUDA_OK;
}

int loom_gguf_resolve(const loom_gguf *g, const char *name, loom_gguf_view *out) {
    const Info *t = g->find_tensor(name);
    if (!t) return g_gguf_err = "MissingTensor", LOOM_CUDA_DECLINED;
    uint64_t be, bb;
    type_geom(t->type, &be, &bb);
    if (bb == 0) return g_gguf_err = "UnsupportedTensorType", LOOM_CUDA_DECLINED;
    const uint64_t ne0 = t->dims[0];
    const uint64_t ne1 = t->n_dims > 1 ? t->dims[1] : 1;
    const uint64_t ne2 = t->n_dims > 2 ? t->dims[2] : 1;
    // tensorBytesChecked: whole blocks per row, every product overflow-checked
    if (be != 1 && ne0 % be != 0) return g_gguf_err = "BadTensorShape", LOOM_CUDA_DECLINED;
    uint64_t row, slice, bytes;
    if (mul_ovf(ne0 / be, bb, &row) || mul_ovf(ne1, row, &slice) || mul_ovf(slice, ne2, &bytes))
        return g_gguf_err = "BadTensorShape", LOOM_CUDA_DECLINED;
    uint64_t start, end;
    if (add_ovf(g->data_offset, t->offset, &start) || add_ovf(start, bytes, &end) || end > g->size)
        return g_gguf_err = "TruncatedGguf", LOOM_CUDA_DECLINED;
    out->ggml_type = (int)t->type;
    out->data = g->image + start;
    out->bytes = (size_t)bytes;
    out->ne0 = ne0;
    out->ne1 = ne1;
    out->ne2 = ne2;
    g_gguf_err.clear();
    return LOOM_CUDA_OK;
}

}  // extern "C"
