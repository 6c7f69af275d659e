// safetensors.cpp -- the st_* reader (include/safetensors.h), host side, load time.
//
// Format: bytes 0..7 hold the header length N (unsigned 64-bit little endian),
// bytes 8..8+N-1 a JSON object, the rest is the data segment. Each member other
// than "__metadata__" is {"dtype": str, "shape": [uint...], "data_offsets":
// [begin, end]} with offsets relative to the data segment. The parser accepts
// objects, arrays, strings (with the simple escapes) and unsigned integers,
// skips unknown keys inside a tensor object, and rejects anything else: the
// same accepted subset as the reference reader (src/safetensors.c:1-33).
#include "../../include/safetensors.h"

#include <cerrno>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

struct st_file {
    FILE* fp = nullptr;
    uint64_t file_size = 0, header_length = 0, data_offset = 0;
    std::vector<st_tensor> tensors;
    std::vector<std::pair<std::string, std::string>> meta;
    int has_metadata = 0;
};

namespace {

struct DT { const char* name; st_dtype d; size_t size; };
const DT kDtypes[] = {
    {"BOOL", ST_DTYPE_BOOL, 1}, {"U8", ST_DTYPE_U8, 1},     {"I8", ST_DTYPE_I8, 1},
    {"U16", ST_DTYPE_U16, 2},   {"I16", ST_DTYPE_I16, 2},   {"F16", ST_DTYPE_F16, 2},
    {"BF16", ST_DTYPE_BF16, 2}, {"U32", ST_DTYPE_U32, 4},   {"I32", ST_DTYPE_I32, 4},
    {"F32", ST_DTYPE_F32, 4},   {"U64", ST_DTYPE_U64, 8},   {"I64", ST_DTYPE_I64, 8},
    {"F64", ST_DTYPE_F64, 8}};

struct Parser {
    const char* p;
    const char* end;
    void ws() { while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p; }
    bool eat(char c) { ws(); if (p < end && *p == c) { ++p; return true; } return false; }
    bool peek(char c) { ws(); return p < end && *p == c; }
    bool str(std::string& out) {
        ws();
        if (p >= end || *p != '"') return false;
        ++p;
        out.clear();
        while (p < end && *p != '"') {
            char c = *p++;
            if (c == '\\') {
                if (p >= end) return false;
                char e = *p++;
                switch (e) {
                    case '"': c = '"'; break;
                    case '\\': c = '\\'; break;
                    case '/': c = '/'; break;
                    case 'b': c = '\b'; break;
                    case 'f': c = '\f'; break;
                    case 'n': c = '\n'; break;
                    case 'r': c = '\r'; break;
                    case 't': c = '\t'; break;
                    default: return false;  // \uXXXX and the rest are refused
                }
            }
            out.push_back(c);
        }
        if (p >= end) return false;
        ++p;
        return true;
    }
    bool uint(uint64_t& v) {
        ws();
        if (p >= end || *p < '0' || *p > '9') return false;
        v = 0;
        while (p < end && *p >= '0' && *p <= '9') {
            const uint64_t d = (uint64_t)(*p - '0');
            if (v > (UINT64_MAX - d) / 10) return false;
            v = v * 10 + d;
            ++p;
        }
        return !(p < end && (*p == '.' || *p == 'e' || *p == 'E'));
    }
    // skips any accepted value (used for unknown keys)
    bool skip() {
        ws();
        if (p >= end) return false;
        if (*p == '"') { std::string s; return str(s); }
        if (*p >= '0' && *p <= '9') { uint64_t v; return uint(v); }
        if (eat('[')) {
            if (eat(']')) return true;
            do { if (!skip()) return false; } while (eat(','));
            return eat(']');
        }
        if (eat('{')) {
            if (eat('}')) return true;
            do { std::string k; if (!str(k) || !eat(':') || !skip()) return false; } while (eat(','));
            return eat('}');
        }
        return false;
    }
};

st_status parse_header(st_file* f, const char* text, size_t n) {
    Parser ps{text, text + n};
    if (!ps.eat('{')) return ST_ERR_BAD_JSON;
    if (ps.eat('}')) { ps.ws(); return ps.p == ps.end ? ST_OK : ST_ERR_BAD_JSON; }
    const uint64_t data_bytes = f->file_size - f->data_offset;
    do {
        std::string name;
        if (!ps.str(name) || !ps.eat(':')) return ST_ERR_BAD_JSON;
        if (name == "__metadata__") {
            if (!ps.eat('{')) return ST_ERR_BAD_JSON;
            f->has_metadata = 1;
            if (!ps.eat('}')) {
                do {
                    std::string k, v;
                    if (!ps.str(k) || !ps.eat(':') || !ps.str(v)) return ST_ERR_BAD_JSON;
                    f->meta.emplace_back(k, v);
                } while (ps.eat(','));
                if (!ps.eat('}')) return ST_ERR_BAD_JSON;
            }
            continue;
        }
        if (name.size() >= ST_MAX_NAME) return ST_ERR_NAME_TOO_LONG;
        st_tensor t;
        std::memset(&t, 0, sizeof t);
        std::memcpy(t.name, name.c_str(), name.size() + 1);
        bool have_dtype = false, have_shape = false, have_off = false;
        if (!ps.eat('{')) return ST_ERR_BAD_JSON;
        do {
            std::string key;
            if (!ps.str(key) || !ps.eat(':')) return ST_ERR_BAD_JSON;
            if (key == "dtype") {
                std::string d;
                if (have_dtype || !ps.str(d)) return ST_ERR_BAD_JSON;
                t.dtype = ST_DTYPE_UNKNOWN;
                for (const DT& e : kDtypes) if (d == e.name) t.dtype = e.d;
                if (t.dtype == ST_DTYPE_UNKNOWN) return ST_ERR_BAD_DTYPE;
                have_dtype = true;
            } else if (key == "shape") {
                if (have_shape || !ps.eat('[')) return ST_ERR_BAD_JSON;
                if (!ps.eat(']')) {
                    do {
                        uint64_t v;
                        if (!ps.uint(v)) return ST_ERR_BAD_SHAPE;
                        if (t.n_dims >= ST_MAX_DIMS) return ST_ERR_TOO_MANY_DIMS;
                        t.dims[t.n_dims++] = (int64_t)v;
                    } while (ps.eat(','));
                    if (!ps.eat(']')) return ST_ERR_BAD_JSON;
                }
                have_shape = true;
            } else if (key == "data_offsets") {
                if (have_off || !ps.eat('[') || !ps.uint(t.begin) || !ps.eat(',') ||
                    !ps.uint(t.end) || !ps.eat(']'))
                    return ST_ERR_BAD_JSON;
                have_off = true;
            } else if (!ps.skip()) {
                return ST_ERR_BAD_JSON;
            }
        } while (ps.eat(','));
        if (!ps.eat('}')) return ST_ERR_BAD_JSON;
        if (!have_dtype || !have_off) return ST_ERR_BAD_JSON;
        if (!have_shape) return ST_ERR_BAD_SHAPE;
        if (t.end < t.begin || t.end > data_bytes) return ST_ERR_RANGE;
        t.nbytes = t.end - t.begin;
        t.file_offset = f->data_offset + t.begin;
        uint64_t elems = 1;
        for (int i = 0; i < t.n_dims; ++i) elems *= (uint64_t)t.dims[i];
        if (elems * st_dtype_size(t.dtype) != t.nbytes) return ST_ERR_SIZE_MISMATCH;
        f->tensors.push_back(t);
    } while (ps.eat(','));
    if (!ps.eat('}')) return ST_ERR_BAD_JSON;
    ps.ws();
    return ps.p == ps.end ? ST_OK : ST_ERR_BAD_JSON;
}

}  // namespace

extern "C" {

size_t st_dtype_size(st_dtype d) {
    for (const DT& e : kDtypes) if (e.d == d) return e.size;
    return 0;
}

const char* st_dtype_name(st_dtype d) {
    for (const DT& e : kDtypes) if (e.d == d) return e.name;
    return "UNKNOWN";
}

const char* st_strerror(st_status s) {
    switch (s) {
        case ST_OK: return "ok";
        case ST_ERR_OPEN: return "the weight file could not be opened";
        case ST_ERR_READ: return "a read failed or came back short";
        case ST_ERR_TRUNCATED_HEADER: return "the declared header runs past the end of the file";
        case ST_ERR_BAD_JSON: return "the header is outside the accepted JSON subset";
        case ST_ERR_BAD_DTYPE: return "a dtype spelling is not recognised";
        case ST_ERR_BAD_SHAPE: return "a shape is missing or malformed";
        case ST_ERR_RANGE: return "a tensor's byte range leaves the data segment";
        case ST_ERR_SIZE_MISMATCH: return "a tensor's byte length disagrees with its shape and dtype";
        case ST_ERR_NOT_FOUND: return "no tensor of that name";
        case ST_ERR_TOO_MANY_DIMS: return "a shape has more dimensions than supported";
        case ST_ERR_NAME_TOO_LONG: return "a tensor name is too long";
        case ST_ERR_NOMEM: return "allocation failed";
        case ST_ERR_ARG: return "a null or unusable argument";
    }
    return "unknown";
}

st_status st_open(const char* path, st_file** out) {
    if (!path || !out) return ST_ERR_ARG;
    *out = nullptr;
    FILE* fp = std::fopen(path, "rb");
    if (!fp) return ST_ERR_OPEN;
    st_file* f = new (std::nothrow) st_file();
    if (!f) { std::fclose(fp); return ST_ERR_NOMEM; }
    f->fp = fp;
    unsigned char len8[8];
    st_status rc = ST_OK;
    std::vector<char> hdr;
    if (fseeko(fp, 0, SEEK_END) != 0) { rc = ST_ERR_READ; goto fail; }
    f->file_size = (uint64_t)ftello(fp);
    if (fseeko(fp, 0, SEEK_SET) != 0 || std::fread(len8, 1, 8, fp) != 8) { rc = ST_ERR_TRUNCATED_HEADER; goto fail; }
    f->header_length = 0;
    for (int i = 7; i >= 0; --i) f->header_length = (f->header_length << 8) | len8[i];
    if (f->header_length > f->file_size - 8) { rc = ST_ERR_TRUNCATED_HEADER; goto fail; }
    f->data_offset = 8 + f->header_length;
    hdr.resize((size_t)f->header_length);
    if (f->header_length &&
        std::fread(hdr.data(), 1, (size_t)f->header_length, fp) != (size_t)f->header_length) {
        rc = ST_ERR_READ;
        goto fail;
    }
    rc = parse_header(f, hdr.data(), hdr.size());
    if (rc != ST_OK) goto fail;
    *out = f;
    return ST_OK;
fail:
    st_close(f);
    return rc;
}

void st_close(st_file* f) {
    if (!f) return;
    if (f->fp) std::fclose(f->fp);
    delete f;
}

size_t st_count(const st_file* f) { return f ? f->tensors.size() : 0; }

const st_tensor* st_at(const st_file* f, size_t i) {
    return (f && i < f->tensors.size()) ? &f->tensors[i] : nullptr;
}

st_status st_find(const st_file* f, const char* name, const st_tensor** out) {
    if (!f || !name || !out) return ST_ERR_ARG;
    for (const st_tensor& t : f->tensors)
        if (std::strcmp(t.name, name) == 0) { *out = &t; return ST_OK; }
    *out = nullptr;
    return ST_ERR_NOT_FOUND;
}

st_status st_tensor_read(const st_file* f, const st_tensor* t, void* dst, size_t dst_bytes) {
    if (!f || !t || (!dst && t->nbytes)) return ST_ERR_ARG;
    if (dst_bytes < t->nbytes) return ST_ERR_ARG;
    if (fseeko(f->fp, (off_t)t->file_offset, SEEK_SET) != 0) return ST_ERR_READ;
    if (t->nbytes && std::fread(dst, 1, (size_t)t->nbytes, f->fp) != (size_t)t->nbytes) return ST_ERR_READ;
    return ST_OK;
}

uint64_t st_header_length(const st_file* f) { return f ? f->header_length : 0; }
uint64_t st_data_offset(const st_file* f) { return f ? f->data_offset : 0; }
uint64_t st_file_size(const st_file* f) { return f ? f->file_size : 0; }

const char* st_metadata(const st_file* f, const char* key) {
    if (!f || !key) return nullptr;
    for (const auto& kv : f->meta) if (kv.first == key) return kv.second.c_str();
    return nullptr;
}

int st_has_metadata(const st_file* f) { return f ? f->has_metadata : 0; }

}  // extern "C"

namespace tie {

// Bytes [offset, offset + n) of tensor t's data into dst (the loader streams a
// tensor through pinned staging buffers this way).
st_status st_tensor_read_range(const st_file* f, const st_tensor* t, uint64_t offset, void* dst, size_t n) {
    if (!f || !t || (!dst && n)) return ST_ERR_ARG;
    if (offset > t->nbytes || n > t->nbytes - offset) return ST_ERR_ARG;
    if (fseeko(f->fp, (off_t)(t->file_offset + offset), SEEK_SET) != 0) return ST_ERR_READ;
    if (n && std::fread(dst, 1, n, f->fp) != n) return ST_ERR_READ;
    return ST_OK;
}

}  // namespace tie
