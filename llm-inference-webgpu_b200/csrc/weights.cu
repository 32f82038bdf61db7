// Safetensors reader (include/b2a.h, b2a_safetensors_*): Safetensors.open /
// info / readRaw / readF32 of src/core/safetensors.js:36-199, host code. The
// header is parsed with st_json and validated in the reference's order with
// its messages; tensor bytes are read on demand with pread (files) or from a
// private copy (memory images).
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "b2a_internal.cuh"
#include "st_json.h"

struct b2a_safetensors {
  int fd = -1;                       // file source, or
  std::vector<unsigned char> mem;    // memory source
  uint64_t file_size = 0, data_start = 0;
  struct Tensor {
    std::string name, dtype;
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0;     // offsets into the data section
  };
  std::vector<Tensor> tensors;       // header order
  bool has_metadata = false;
  std::string metadata;              // the __metadata__ value as JSON text
};

using namespace b2a;

namespace {

// Bytes per element of the dtypes safetensors defines (safetensors.js:15-20).
int dtype_bytes(const std::string& d) {
  static const struct { const char* name; int bytes; } kTable[] = {
      {"BOOL", 1}, {"U8", 1},  {"I8", 1},  {"F8_E4M3", 1}, {"F8_E5M2", 1}, {"I16", 2}, {"U16", 2}, {"F16", 2},
      {"BF16", 2}, {"I32", 4}, {"U32", 4}, {"F32", 4},     {"I64", 8},     {"U64", 8}, {"F64", 8}};
  for (const auto& e : kTable)
    if (d == e.name) return e.bytes;
  return 0;
}

// A JavaScript number as a template literal prints it: integers in plain
// digits, others in their shortest round-trip form.
std::string js_number(double v) {
  char buf[64];
  if (std::isnan(v)) return "NaN";
  if (std::isinf(v)) return v > 0 ? "Infinity" : "-Infinity";
  if (v == std::floor(v) && std::fabs(v) < 1e21) {
    snprintf(buf, sizeof(buf), "%.0f", v);
    return buf;
  }
  for (int prec = 1; prec <= 17; prec++) {
    snprintf(buf, sizeof(buf), "%.*g", prec, v);
    if (std::strtod(buf, nullptr) == v) break;
  }
  return buf;
}

// JSON.stringify of a header value (for the unknown-dtype message).
std::string js_stringify(const json::Value* v, const std::string& text) {
  if (v == nullptr) return "undefined";
  if (v->kind == json::Value::String) return "\"" + v->str + "\"";
  return text.substr(v->begin, v->end - v->begin);
}

bool safe_integer(double v) { return std::isfinite(v) && v == std::floor(v) && std::fabs(v) <= 9007199254740991.0; }

bool read_at(const b2a_safetensors* st, uint64_t off, void* dst, size_t n) {
  if (st->fd < 0) {
    if (off + n > st->mem.size()) return false;
    std::memcpy(dst, st->mem.data() + off, n);
    return true;
  }
  auto* p = static_cast<unsigned char*>(dst);
  while (n > 0) {
    const ssize_t got = pread(st->fd, p, n, static_cast<off_t>(off));
    if (got <= 0) return false;
    p += got;
    off += static_cast<uint64_t>(got);
    n -= static_cast<size_t>(got);
  }
  return true;
}

b2a_status parse_header(b2a_safetensors* st) {
  const uint64_t size = st->file_size;
  if (size < 8) return fail(B2A_EINVAL, "not a safetensors file: %llu bytes", static_cast<unsigned long long>(size));
  unsigned char lenb[8];
  if (!read_at(st, 0, lenb, 8)) return fail(B2A_EINVAL, "could not read the header length");
  uint64_t hl = 0;
  for (int k = 7; k >= 0; k--) hl = (hl << 8) | lenb[k];
  const double hlen = static_cast<double>(hl);   // Number(BigInt)
  if (!safe_integer(hlen) || hlen <= 0 || 8.0 + hlen > static_cast<double>(size)) {
    return fail(B2A_EINVAL, "header length %s does not fit in a %llu-byte file", js_number(hlen).c_str(),
                static_cast<unsigned long long>(size));
  }
  std::string text(static_cast<size_t>(hl), '\0');
  if (!read_at(st, 8, &text[0], text.size())) return fail(B2A_EINVAL, "could not read the header");
  json::Value header;
  std::string err;
  if (!json::parse(text.data(), text.size(), &header, &err)) {
    return fail(B2A_EINVAL, "header is not valid UTF-8 JSON: %s", err.c_str());
  }
  if (header.kind != json::Value::Object) return fail(B2A_EINVAL, "header must be a JSON object");

  st->data_start = 8 + hl;
  const double data_size = static_cast<double>(size - st->data_start);
  for (const auto& m : header.members) {
    const std::string& name = m.first;
    const json::Value& entry = m.second;
    if (name == "__metadata__") {
      if (entry.kind != json::Value::Null) {   // `header.__metadata__ ?? null`
        st->has_metadata = true;
        st->metadata = text.substr(entry.begin, entry.end - entry.begin);
      }
      continue;
    }
    const bool obj = entry.kind == json::Value::Object;
    const json::Value* dt = obj ? entry.get("dtype") : nullptr;
    const json::Value* shape = obj ? entry.get("shape") : nullptr;
    const json::Value* offs = obj ? entry.get("data_offsets") : nullptr;
    const int esz = (dt && dt->kind == json::Value::String) ? dtype_bytes(dt->str) : 0;
    if (esz == 0) return fail(B2A_EINVAL, "%s: unknown dtype %s", name.c_str(), js_stringify(dt, text).c_str());
    bool shape_ok = shape && shape->kind == json::Value::Array;
    if (shape_ok) {
      for (const auto& d : shape->items) shape_ok &= d.kind == json::Value::Number && safe_integer(d.num) && d.num >= 0;
    }
    if (!shape_ok) return fail(B2A_EINVAL, "%s: shape must be an array of non-negative integers", name.c_str());
    if (!offs || offs->kind != json::Value::Array || offs->items.size() != 2) {
      return fail(B2A_EINVAL, "%s: data_offsets must be a pair", name.c_str());
    }
    const json::Value& vb = offs->items[0];
    const json::Value& ve = offs->items[1];
    const bool nums = vb.kind == json::Value::Number && ve.kind == json::Value::Number;
    const double b = nums ? vb.num : NAN, e = nums ? ve.num : NAN;
    if (!nums || !safe_integer(b) || !safe_integer(e) || b < 0 || e < b) {
      const std::string sb = vb.kind == json::Value::Number ? js_number(vb.num) : js_stringify(&vb, text);
      const std::string se = ve.kind == json::Value::Number ? js_number(ve.num) : js_stringify(&ve, text);
      return fail(B2A_EINVAL, "%s: bad data_offsets [%s, %s]", name.c_str(), sb.c_str(), se.c_str());
    }
    if (e > data_size) {
      return fail(B2A_EINVAL, "%s: ends at %s but the data section is only %s bytes", name.c_str(),
                  js_number(e).c_str(), js_number(data_size).c_str());
    }
    double numel = 1.0;
    std::string dims;
    b2a_safetensors::Tensor t;
    for (size_t k = 0; k < shape->items.size(); k++) {
      numel *= shape->items[k].num;
      dims += (k ? "," : "") + js_number(shape->items[k].num);
      t.shape.push_back(static_cast<int64_t>(shape->items[k].num));
    }
    if (e - b != numel * esz) {
      return fail(B2A_EINVAL, "%s: shape [%s] of %s needs %s bytes but the header reserves %s", name.c_str(),
                  dims.c_str(), dt->str.c_str(), js_number(numel * esz).c_str(), js_number(e - b).c_str());
    }
    t.name = name;
    t.dtype = dt->str;
    t.begin = static_cast<uint64_t>(b);
    t.end = static_cast<uint64_t>(e);
    st->tensors.push_back(std::move(t));
  }
  // overlapping ranges (safetensors.js:115-121): sorted by start, stable
  std::vector<const b2a_safetensors::Tensor*> ranges;
  for (const auto& t : st->tensors) ranges.push_back(&t);
  std::stable_sort(ranges.begin(), ranges.end(),
                   [](const b2a_safetensors::Tensor* a, const b2a_safetensors::Tensor* b) { return a->begin < b->begin; });
  for (size_t i = 1; i < ranges.size(); i++) {
    if (ranges[i]->begin < ranges[i - 1]->end) {
      return fail(B2A_EINVAL, "%s overlaps %s", ranges[i]->name.c_str(), ranges[i - 1]->name.c_str());
    }
  }
  return B2A_OK;
}

const b2a_safetensors::Tensor* find(const b2a_safetensors* st, const char* name) {
  for (const auto& t : st->tensors)
    if (t.name == name) return &t;
  return nullptr;
}

// f16 bits -> f32, exactly (src/core/dtype.js:55-78)
float f16_to_f32(uint16_t h) {
  const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {   // subnormal: man * 2^-24, exact in f32
      float f = std::ldexp(static_cast<float>(man), -24);
      std::memcpy(&bits, &f, 4);
      bits |= sign;
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112) << 23) | (man << 13);
  }
  float out;
  std::memcpy(&out, &bits, 4);
  return out;
}

}  // namespace

namespace b2a {

// The tensor's bytes [offset, offset + length) (readRawRange, safetensors.js:148-156).
b2a_status st_read_range(const b2a_safetensors* st, const char* name, uint64_t offset, uint64_t length, void* dst) {
  const b2a_safetensors::Tensor* t = find(st, name);
  if (t == nullptr) return fail(B2A_EINVAL, "no tensor named \"%s\"", name);
  if (offset + length > t->end - t->begin) {
    return fail(B2A_ERANGE, "%s: range %llu+%llu outside a %llu-byte tensor", name,
                static_cast<unsigned long long>(offset), static_cast<unsigned long long>(length),
                static_cast<unsigned long long>(t->end - t->begin));
  }
  if (!read_at(st, st->data_start + t->begin + offset, dst, static_cast<size_t>(length))) {
    return fail(B2A_EINVAL, "%s: could not read %llu bytes", name, static_cast<unsigned long long>(length));
  }
  return B2A_OK;
}

// n elements of dtype `dt` at src -> f32 (readF32's widening, safetensors.js:166-193).
bool st_widen(const std::string& dt, const void* src, size_t n, float* dst) {
  if (dt == "F32") {
    std::memcpy(dst, src, n * 4);
  } else if (dt == "BF16") {
    const auto* s = static_cast<const uint16_t*>(src);
    for (size_t i = 0; i < n; i++) {
      const uint32_t bits = static_cast<uint32_t>(s[i]) << 16;
      std::memcpy(dst + i, &bits, 4);
    }
  } else if (dt == "F16") {
    const auto* s = static_cast<const uint16_t*>(src);
    for (size_t i = 0; i < n; i++) dst[i] = f16_to_f32(s[i]);
  } else if (dt == "F64") {
    const auto* s = static_cast<const double*>(src);
    for (size_t i = 0; i < n; i++) dst[i] = static_cast<float>(s[i]);
  } else {
    return false;
  }
  return true;
}

}  // namespace b2a

extern "C" {

b2a_status b2a_safetensors_open(const char* path, b2a_safetensors** out) {
  if (path == nullptr || out == nullptr) return fail(B2A_EINVAL, "null argument");
  *out = nullptr;
  auto* st = new (std::nothrow) b2a_safetensors();
  if (st == nullptr) return fail(B2A_EINVAL, "out of host memory");
  st->fd = open(path, O_RDONLY | O_CLOEXEC);
  struct stat sb;
  if (st->fd < 0 || fstat(st->fd, &sb) != 0) {
    const int e = errno;
    if (st->fd >= 0) close(st->fd);
    delete st;
    return fail(B2A_EINVAL, "cannot open %s: %s", path, std::strerror(e));
  }
  st->file_size = static_cast<uint64_t>(sb.st_size);
  const b2a_status s = parse_header(st);
  if (s != B2A_OK) {
    close(st->fd);
    delete st;
    return s;
  }
  *out = st;
  return B2A_OK;
}

b2a_status b2a_safetensors_open_memory(const void* bytes, size_t size, b2a_safetensors** out) {
  if ((bytes == nullptr && size > 0) || out == nullptr) return fail(B2A_EINVAL, "null argument");
  *out = nullptr;
  auto* st = new (std::nothrow) b2a_safetensors();
  if (st == nullptr) return fail(B2A_EINVAL, "out of host memory");
  try {
    st->mem.assign(static_cast<const unsigned char*>(bytes), static_cast<const unsigned char*>(bytes) + size);
  } catch (...) {
    delete st;
    return fail(B2A_EINVAL, "out of host memory");
  }
  st->file_size = size;
  const b2a_status s = parse_header(st);
  if (s != B2A_OK) {
    delete st;
    return s;
  }
  *out = st;
  return B2A_OK;
}

b2a_status b2a_safetensors_close(b2a_safetensors* st) {
  if (st == nullptr) return B2A_OK;
  if (st->fd >= 0) close(st->fd);
  delete st;
  return B2A_OK;
}

int b2a_safetensors_count(const b2a_safetensors* st) { return st ? static_cast<int>(st->tensors.size()) : 0; }

const char* b2a_safetensors_name(const b2a_safetensors* st, int index) {
  if (st == nullptr || index < 0 || index >= static_cast<int>(st->tensors.size())) return nullptr;
  return st->tensors[index].name.c_str();
}

const char* b2a_safetensors_metadata(const b2a_safetensors* st) {
  return (st && st->has_metadata) ? st->metadata.c_str() : nullptr;
}

b2a_status b2a_safetensors_info(const b2a_safetensors* st, const char* name, char* dtype, int64_t* shape,
                                int max_dims, int* ndim, int64_t* byte_length) {
  if (st == nullptr || name == nullptr) return fail(B2A_EINVAL, "null argument");
  const b2a_safetensors::Tensor* t = find(st, name);
  if (t == nullptr) return fail(B2A_EINVAL, "no tensor named \"%s\"", name);   // safetensors.js:127-131
  if (dtype) snprintf(dtype, 16, "%s", t->dtype.c_str());
  if (ndim) *ndim = static_cast<int>(t->shape.size());
  if (shape) {
    for (int k = 0; k < max_dims && k < static_cast<int>(t->shape.size()); k++) shape[k] = t->shape[k];
  }
  if (byte_length) *byte_length = static_cast<int64_t>(t->end - t->begin);
  return B2A_OK;
}

b2a_status b2a_safetensors_read_raw(const b2a_safetensors* st, const char* name, void* dst, size_t capacity) {
  if (st == nullptr || name == nullptr) return fail(B2A_EINVAL, "null argument");
  const b2a_safetensors::Tensor* t = find(st, name);
  if (t == nullptr) return fail(B2A_EINVAL, "no tensor named \"%s\"", name);
  const uint64_t n = t->end - t->begin;
  if (capacity < n || (dst == nullptr && n > 0)) {
    return fail(B2A_EINVAL, "%s: needs %llu bytes of room, got %zu", name, static_cast<unsigned long long>(n), capacity);
  }
  return st_read_range(st, name, 0, n, dst);
}

b2a_status b2a_safetensors_read_f32(const b2a_safetensors* st, const char* name, float* dst, size_t count) {
  if (st == nullptr || name == nullptr) return fail(B2A_EINVAL, "null argument");
  const b2a_safetensors::Tensor* t = find(st, name);
  if (t == nullptr) return fail(B2A_EINVAL, "no tensor named \"%s\"", name);
  const int esz = dtype_bytes(t->dtype);
  const uint64_t n = (t->end - t->begin) / static_cast<uint64_t>(esz);
  const std::string& dt = t->dtype;
  if (dt != "F32" && dt != "BF16" && dt != "F16" && dt != "F64") {
    return fail(B2A_EINVAL, "%s: cannot widen %s to f32", name, dt.c_str());
  }
  if (count < n || (dst == nullptr && n > 0)) {
    return fail(B2A_EINVAL, "%s: needs room for %llu floats, got %zu", name, static_cast<unsigned long long>(n), count);
  }
  // in blocks, so a large bf16 tensor never needs a full-size staging copy
  constexpr uint64_t kBlock = 1 << 20;   // elements
  std::vector<unsigned char> buf(static_cast<size_t>(std::min<uint64_t>(n, kBlock) * esz));
  for (uint64_t i = 0; i < n; i += kBlock) {
    const uint64_t m = std::min<uint64_t>(kBlock, n - i);
    const b2a_status s = st_read_range(st, name, i * esz, m * esz, buf.data());
    if (s != B2A_OK) return s;
    st_widen(dt, buf.data(), static_cast<size_t>(m), dst + i);
  }
  return B2A_OK;
}

}  // extern "C"
