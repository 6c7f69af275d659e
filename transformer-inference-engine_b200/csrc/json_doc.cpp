// json_doc.cpp -- recursive-descent JSON reader into a value tree (json_doc.h).
#include "json_doc.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>

namespace tie {
namespace json {

const Value* Value::get(const std::string& key) const {
    if (kind != Kind::Object) return nullptr;
    for (const auto& m : members)
        if (m.first == key) return &m.second;
    return nullptr;
}

namespace {

constexpr int kMaxDepth = 64;

class Reader {
  public:
    Reader(const char* s, size_t n) : cur_(s), end_(s + n) {}

    bool document(Value* v) {
        if (!value(v, 0)) return false;
        skip_ws();
        return cur_ == end_;
    }

  private:
    const char* cur_;
    const char* end_;

    void skip_ws() {
        while (cur_ < end_ && (*cur_ == ' ' || *cur_ == '\n' || *cur_ == '\r' || *cur_ == '\t')) ++cur_;
    }
    bool literal(const char* word) {
        const size_t n = std::strlen(word);
        if ((size_t)(end_ - cur_) < n || std::memcmp(cur_, word, n) != 0) return false;
        cur_ += n;
        return true;
    }
    static int hex(char c) {
        if (c >= '0' && c <= '9') return c - '0';
        if (c >= 'a' && c <= 'f') return c - 'a' + 10;
        if (c >= 'A' && c <= 'F') return c - 'A' + 10;
        return -1;
    }
    static void put_utf8(std::string& s, unsigned cp) {
        if (cp < 0x80) {
            s.push_back((char)cp);
        } else if (cp < 0x800) {
            s.push_back((char)(0xC0 | (cp >> 6)));
            s.push_back((char)(0x80 | (cp & 0x3F)));
        } else if (cp < 0x10000) {
            s.push_back((char)(0xE0 | (cp >> 12)));
            s.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
            s.push_back((char)(0x80 | (cp & 0x3F)));
        } else {
            s.push_back((char)(0xF0 | (cp >> 18)));
            s.push_back((char)(0x80 | ((cp >> 12) & 0x3F)));
            s.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
            s.push_back((char)(0x80 | (cp & 0x3F)));
        }
    }
    bool hex4(unsigned* cp) {
        if (end_ - cur_ < 4) return false;
        unsigned v = 0;
        for (int i = 0; i < 4; ++i) {
            const int h = hex(cur_[i]);
            if (h < 0) return false;
            v = v * 16 + (unsigned)h;
        }
        cur_ += 4;
        *cp = v;
        return true;
    }
    bool string(std::string* out) {
        if (cur_ >= end_ || *cur_ != '"') return false;
        ++cur_;
        out->clear();
        while (cur_ < end_) {
            const unsigned char c = (unsigned char)*cur_++;
            if (c == '"') return true;
            if (c < 0x20) return false;                 // control characters must be escaped
            if (c != '\\') { out->push_back((char)c); continue; }
            if (cur_ >= end_) return false;
            const char e = *cur_++;
            switch (e) {
                case '"': out->push_back('"'); break;
                case '\\': out->push_back('\\'); break;
                case '/': out->push_back('/'); break;
                case 'b': out->push_back('\b'); break;
                case 'f': out->push_back('\f'); break;
                case 'n': out->push_back('\n'); break;
                case 'r': out->push_back('\r'); break;
                case 't': out->push_back('\t'); break;
                case 'u': {
                    unsigned cp;
                    if (!hex4(&cp)) return false;
                    if (cp >= 0xD800 && cp < 0xDC00) {         // a surrogate pair
                        unsigned lo;
                        if (!literal("\\u") || !hex4(&lo) || lo < 0xDC00 || lo >= 0xE000) return false;
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    } else if (cp >= 0xDC00 && cp < 0xE000) {
                        return false;
                    }
                    put_utf8(*out, cp);
                    break;
                }
                default: return false;
            }
        }
        return false;
    }
    // RFC 8259 number grammar, converted with strtod on a bounded copy
    bool number(double* out) {
        const char* s = cur_;
        const char* p = cur_;
        if (p < end_ && *p == '-') ++p;
        if (p >= end_) return false;
        if (*p == '0') {
            ++p;
        } else if (*p >= '1' && *p <= '9') {
            while (p < end_ && *p >= '0' && *p <= '9') ++p;
        } else {
            return false;
        }
        if (p < end_ && *p == '.') {
            ++p;
            if (p >= end_ || *p < '0' || *p > '9') return false;
            while (p < end_ && *p >= '0' && *p <= '9') ++p;
        }
        if (p < end_ && (*p == 'e' || *p == 'E')) {
            ++p;
            if (p < end_ && (*p == '+' || *p == '-')) ++p;
            if (p >= end_ || *p < '0' || *p > '9') return false;
            while (p < end_ && *p >= '0' && *p <= '9') ++p;
        }
        const std::string text(s, p);
        *out = std::strtod(text.c_str(), nullptr);
        cur_ = p;
        return true;
    }
    bool value(Value* v, int depth) {
        if (depth > kMaxDepth) return false;
        skip_ws();
        if (cur_ >= end_) return false;
        switch (*cur_) {
            case '{': {
                ++cur_;
                v->kind = Kind::Object;
                skip_ws();
                if (cur_ < end_ && *cur_ == '}') { ++cur_; return true; }
                for (;;) {
                    skip_ws();
                    std::pair<std::string, Value> m;
                    if (!string(&m.first)) return false;
                    skip_ws();
                    if (cur_ >= end_ || *cur_++ != ':') return false;
                    if (!value(&m.second, depth + 1)) return false;
                    v->members.push_back(std::move(m));
                    skip_ws();
                    if (cur_ >= end_) return false;
                    const char c = *cur_++;
                    if (c == '}') return true;
                    if (c != ',') return false;
                }
            }
            case '[': {
                ++cur_;
                v->kind = Kind::Array;
                skip_ws();
                if (cur_ < end_ && *cur_ == ']') { ++cur_; return true; }
                for (;;) {
                    v->items.emplace_back();
                    if (!value(&v->items.back(), depth + 1)) return false;
                    skip_ws();
                    if (cur_ >= end_) return false;
                    const char c = *cur_++;
                    if (c == ']') return true;
                    if (c != ',') return false;
                }
            }
            case '"':
                v->kind = Kind::String;
                return string(&v->str);
            case 't':
                v->kind = Kind::Bool;
                v->b = true;
                return literal("true");
            case 'f':
                v->kind = Kind::Bool;
                v->b = false;
                return literal("false");
            case 'n':
                v->kind = Kind::Null;
                return literal("null");
            default:
                v->kind = Kind::Number;
                return number(&v->num);
        }
    }
};

}  // namespace

bool parse(const char* text, size_t n, Value* out) {
    *out = Value();
    Reader r(text, n);
    return r.document(out);
}

bool read_file(const char* path, std::string* out) {
    FILE* f = std::fopen(path, "rb");
    if (!f) return false;
    out->clear();
    char buf[1 << 16];
    size_t got;
    while ((got = std::fread(buf, 1, sizeof buf, f)) > 0) out->append(buf, got);
    const bool ok = !std::ferror(f);
    std::fclose(f);
    return ok;
}

}  // namespace json
}  // namespace tie
