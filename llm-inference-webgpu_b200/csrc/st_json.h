// A small JSON reader for safetensors headers (host code): objects keep their
// keys in document order, numbers are IEEE doubles (a JavaScript number), the
// input must be well-formed UTF-8 (the reference decodes the header with a
// fatal UTF-8 decoder, src/core/safetensors.js:66-71). A later duplicate key
// replaces the earlier value, as JSON.parse does.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <utility>
#include <vector>

namespace b2a {
namespace json {

struct Value {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0.0;
  std::string str;                                   // String
  std::vector<Value> items;                          // Array
  std::vector<std::pair<std::string, Value>> members;  // Object, document order
  size_t begin = 0, end = 0;                         // byte range of the value in the input

  const Value* get(const std::string& key) const {
    for (const auto& m : members)
      if (m.first == key) return &m.second;
    return nullptr;
  }
};

// Parses text[0, n) as one JSON value (surrounding whitespace allowed).
// On failure returns false and a message like JSON.parse's in *err.
bool parse(const char* text, size_t n, Value* out, std::string* err);

}  // namespace json
}  // namespace b2a
