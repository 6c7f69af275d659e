// json_doc.h -- a small JSON document model for the two load-time text
// artifacts (config.json and the tensor inventory).
//
// The whole text is parsed into a tree first (RFC 8259 values: object, array,
// string, number, true/false/null), then fields are looked up by path. A text
// that is not one well-formed JSON value is rejected as a whole, so a
// truncated or hand-damaged artifact is refused rather than half-read.
#pragma once

#include <map>
#include <memory>
#include <string>
#include <vector>

namespace tie {
namespace json {

enum class Kind { Null, Bool, Number, String, Array, Object };

struct Value {
    Kind kind = Kind::Null;
    bool b = false;
    double num = 0.0;
    std::string str;
    std::vector<Value> items;                                    // Array
    std::vector<std::pair<std::string, Value>> members;          // Object, in text order

    // The first member named `key` of an object, or nullptr.
    const Value* get(const std::string& key) const;
    bool is_number() const { return kind == Kind::Number; }
    bool is_string() const { return kind == Kind::String; }
};

// Parses `text` (n bytes). Returns false, leaving *out unspecified, unless the
// text holds exactly one JSON value with nothing but whitespace around it.
bool parse(const char* text, size_t n, Value* out);

// Reads a whole file; false if it cannot be opened or read.
bool read_file(const char* path, std::string* out);

}  // namespace json
}  // namespace tie
