// JSON reader for safetensors headers (st_json.h). Host code only.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "st_json.h"

namespace b2a {
namespace json {

namespace {

constexpr int kMaxDepth = 128;

struct Parser {
  const char* s;
  size_t n, i = 0;
  std::string err;

  bool fail(const char* what) {
    char buf[160];
    if (i < n) snprintf(buf, sizeof(buf), "%s at position %zu", what, i);
    else snprintf(buf, sizeof(buf), "%s at the end of the input", what);
    err = buf;
    return false;
  }
  void ws() {
    while (i < n && (s[i] == ' ' || s[i] == '\t' || s[i] == '\n' || s[i] == '\r')) i++;
  }
  static void put_utf8(std::string& o, uint32_t cp) {
    if (cp < 0x80) {
      o += static_cast<char>(cp);
    } else if (cp < 0x800) {
      o += static_cast<char>(0xC0 | (cp >> 6));
      o += static_cast<char>(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      o += static_cast<char>(0xE0 | (cp >> 12));
      o += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
      o += static_cast<char>(0x80 | (cp & 0x3F));
    } else {
      o += static_cast<char>(0xF0 | (cp >> 18));
      o += static_cast<char>(0x80 | ((cp >> 12) & 0x3F));
      o += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
      o += static_cast<char>(0x80 | (cp & 0x3F));
    }
  }
  bool hex4(uint32_t* v) {
    if (i + 4 > n) return fail("Bad Unicode escape");
    uint32_t r = 0;
    for (int k = 0; k < 4; k++) {
      const char c = s[i++];
      r <<= 4;
      if (c >= '0' && c <= '9') r |= c - '0';
      else if (c >= 'a' && c <= 'f') r |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') r |= c - 'A' + 10;
      else return fail("Bad Unicode escape");
    }
    *v = r;
    return true;
  }
  bool string(std::string* o) {
    i++;   // the opening quote
    for (;;) {
      if (i >= n) return fail("Unterminated string in JSON");
      const unsigned char c = static_cast<unsigned char>(s[i]);
      if (c == '"') {
        i++;
        return true;
      }
      if (c < 0x20) return fail("Bad control character in string literal");
      if (c != '\\') {
        *o += static_cast<char>(c);
        i++;
        continue;
      }
      i++;
      if (i >= n) return fail("Unterminated string in JSON");
      const char e = s[i++];
      switch (e) {
        case '"': *o += '"'; break;
        case '\\': *o += '\\'; break;
        case '/': *o += '/'; break;
        case 'b': *o += '\b'; break;
        case 'f': *o += '\f'; break;
        case 'n': *o += '\n'; break;
        case 'r': *o += '\r'; break;
        case 't': *o += '\t'; break;
        case 'u': {
          uint32_t cp = 0;
          if (!hex4(&cp)) return false;
          if (cp >= 0xD800 && cp < 0xDC00 && i + 6 <= n && s[i] == '\\' && s[i + 1] == 'u') {
            const size_t save = i;
            i += 2;
            uint32_t lo = 0;
            if (!hex4(&lo)) return false;
            if (lo >= 0xDC00 && lo < 0xE000) cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
            else i = save;   // a lone surrogate, kept as JS keeps it (encoded as is)
          }
          put_utf8(*o, cp);
          break;
        }
        default: return fail("Bad escaped character in JSON");
      }
    }
  }
  bool number(double* v) {
    const size_t b = i;
    if (i < n && s[i] == '-') i++;
    if (i >= n) return fail("No number after minus sign in JSON");
    if (s[i] == '0') {
      i++;
    } else if (s[i] >= '1' && s[i] <= '9') {
      while (i < n && s[i] >= '0' && s[i] <= '9') i++;
    } else {
      return fail("Unexpected token in JSON");
    }
    if (i < n && s[i] == '.') {
      i++;
      if (i >= n || s[i] < '0' || s[i] > '9') return fail("Unterminated fractional number in JSON");
      while (i < n && s[i] >= '0' && s[i] <= '9') i++;
    }
    if (i < n && (s[i] == 'e' || s[i] == 'E')) {
      i++;
      if (i < n && (s[i] == '+' || s[i] == '-')) i++;
      if (i >= n || s[i] < '0' || s[i] > '9') return fail("Exponent part is missing a number in JSON");
      while (i < n && s[i] >= '0' && s[i] <= '9') i++;
    }
    *v = std::strtod(std::string(s + b, i - b).c_str(), nullptr);   // correctly rounded, as JS
    return true;
  }
  bool literal(const char* word) {
    const size_t k = std::strlen(word);
    if (i + k > n || std::memcmp(s + i, word, k) != 0) return fail("Unexpected token in JSON");
    i += k;
    return true;
  }
  bool value(Value* v, int depth) {
    if (depth > kMaxDepth) return fail("JSON nested too deeply");
    ws();
    if (i >= n) return fail("Unexpected end of JSON input");
    v->begin = i;
    const char c = s[i];
    bool ok;
    if (c == '{') {
      v->kind = Value::Object;
      i++;
      ws();
      if (i < n && s[i] == '}') {
        i++;
        ok = true;
      } else {
        ok = false;
        for (;;) {
          ws();
          if (i >= n || s[i] != '"') {
            fail("Expected property name or '}' in JSON");
            break;
          }
          std::string key;
          if (!string(&key)) break;
          ws();
          if (i >= n || s[i] != ':') {
            fail("Expected ':' after property name in JSON");
            break;
          }
          i++;
          Value item;
          if (!value(&item, depth + 1)) break;
          bool replaced = false;
          for (auto& m : v->members) {
            if (m.first == key) {
              m.second = std::move(item);
              replaced = true;
              break;
            }
          }
          if (!replaced) v->members.emplace_back(std::move(key), std::move(item));
          ws();
          if (i < n && s[i] == ',') {
            i++;
            continue;
          }
          if (i < n && s[i] == '}') {
            i++;
            ok = true;
            break;
          }
          fail("Expected ',' or '}' after property value in JSON");
          break;
        }
      }
    } else if (c == '[') {
      v->kind = Value::Array;
      i++;
      ws();
      if (i < n && s[i] == ']') {
        i++;
        ok = true;
      } else {
        ok = false;
        for (;;) {
          Value item;
          if (!value(&item, depth + 1)) break;
          v->items.push_back(std::move(item));
          ws();
          if (i < n && s[i] == ',') {
            i++;
            continue;
          }
          if (i < n && s[i] == ']') {
            i++;
            ok = true;
            break;
          }
          fail("Expected ',' or ']' after array element in JSON");
          break;
        }
      }
    } else if (c == '"') {
      v->kind = Value::String;
      ok = string(&v->str);
    } else if (c == 't') {
      v->kind = Value::Bool;
      v->b = true;
      ok = literal("true");
    } else if (c == 'f') {
      v->kind = Value::Bool;
      ok = literal("false");
    } else if (c == 'n') {
      v->kind = Value::Null;
      ok = literal("null");
    } else {
      v->kind = Value::Number;
      ok = number(&v->num);
    }
    v->end = i;
    return ok;
  }
};

// Well-formed UTF-8 (no overlongs, no surrogates, <= U+10FFFF): what a fatal
// TextDecoder accepts.
bool valid_utf8(const unsigned char* p, size_t n, size_t* bad) {
  size_t i = 0;
  while (i < n) {
    const unsigned c = p[i];
    size_t len;
    uint32_t cp;
    if (c < 0x80) {
      i++;
      continue;
    } else if (c >= 0xC2 && c <= 0xDF) {
      len = 2;
      cp = c & 0x1F;
    } else if (c >= 0xE0 && c <= 0xEF) {
      len = 3;
      cp = c & 0x0F;
    } else if (c >= 0xF0 && c <= 0xF4) {
      len = 4;
      cp = c & 0x07;
    } else {
      *bad = i;
      return false;
    }
    if (i + len > n) {
      *bad = i;
      return false;
    }
    for (size_t k = 1; k < len; k++) {
      if ((p[i + k] & 0xC0) != 0x80) {
        *bad = i;
        return false;
      }
      cp = (cp << 6) | (p[i + k] & 0x3F);
    }
    if ((len == 3 && (cp < 0x800 || (cp >= 0xD800 && cp < 0xE000))) || (len == 4 && (cp < 0x10000 || cp > 0x10FFFF))) {
      *bad = i;
      return false;
    }
    i += len;
  }
  return true;
}

}  // namespace

bool parse(const char* text, size_t n, Value* out, std::string* err) {
  size_t bad = 0;
  if (!valid_utf8(reinterpret_cast<const unsigned char*>(text), n, &bad)) {
    char buf[96];
    snprintf(buf, sizeof(buf), "The encoded data was not valid for encoding utf-8 (byte %zu)", bad);
    *err = buf;
    return false;
  }
  Parser p{text, n};
  if (!p.value(out, 0)) {
    *err = p.err;
    return false;
  }
  p.ws();
  if (p.i != n) {
    p.fail("Unexpected non-whitespace character after JSON");
    *err = p.err;
    return false;
  }
  return true;
}

}  // namespace json
}  // namespace b2a
