// GGUF v2/v3 reader for the engine's own loading path (qc_engine_create_gguf /
// qc_engine_open).  It accepts and rejects files as the reference loader
// src/gguf.rs:102-195 does: header magic and version, count and metadata-budget
// limits, depth-limited arrays, finite floats, strict booleans, single-file
// models, tensor rank 1..3 with non-zero dims, aligned / in-bounds /
// non-overlapping tensor data.
#pragma once
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <cmath>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

#include "layout.h"

namespace qc {

struct GgufError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

struct MetaValue {
  enum Type { Unsigned, Signed, Float, Bool, String, Array } type = Unsigned;
  uint64_t u = 0;
  int64_t i = 0;
  double f = 0;
  std::string s;
  size_t n_items = 0;
  bool get_u64(uint64_t* out) const {  // serde_json as_u64
    if (type == Unsigned) return *out = u, true;
    if (type == Signed && i >= 0) return *out = (uint64_t)i, true;
    return false;
  }
  bool get_f64(double* out) const {  // serde_json as_f64
    if (type == Unsigned) return *out = (double)u, true;
    if (type == Signed) return *out = (double)i, true;
    if (type == Float) return *out = f, true;
    return false;
  }
};

struct GgufTensor {
  std::string name;
  std::vector<uint64_t> dims;
  uint32_t kind = 0;
  uint64_t offset = 0, len = 0;  // absolute offset into the image after parsing
};

class GgufFile {
 public:
  std::map<std::string, MetaValue> meta;
  std::map<std::string, GgufTensor> tensors;

  void parse(const uint8_t* data, uint64_t size) {
    p_ = data;
    n_ = size;
    at_ = 0;
    budget_ = 128ull << 20;
    char magic[4];
    bytes(magic, 4);
    if (memcmp(magic, "GGUF", 4) != 0) throw GgufError("not a GGUF file");
    const uint32_t version = rd<uint32_t>();
    if (version != 2 && version != 3) throw GgufError("GGUF version " + std::to_string(version) + " unsupported");
    const uint64_t nt = count(100000), nk = count(100000);
    for (uint64_t k = 0; k < nk; k++) {
      std::string key = text();
      const uint32_t t = rd<uint32_t>();
      MetaValue v = value(t, 0);
      if (!meta.emplace(std::move(key), std::move(v)).second) throw GgufError("duplicate metadata key");
    }
    uint64_t splits = 1;
    auto sp = meta.find("split.count");
    if (sp != meta.end() && !sp->second.get_u64(&splits)) splits = 1;
    if (splits != 1) throw GgufError("split GGUF not supported; merge shards first");
    for (uint64_t k = 0; k < nt; k++) {
      GgufTensor t;
      t.name = text();
      const uint32_t nd = rd<uint32_t>();
      if (nd < 1 || nd > 3) throw GgufError("unsupported tensor rank " + std::to_string(nd) + ": " + t.name);
      for (uint32_t d = 0; d < nd; d++) {
        const uint64_t dim = rd<uint64_t>();
        if (dim == 0) throw GgufError("zero tensor dimension");
        t.dims.push_back(dim);
      }
      t.kind = rd<uint32_t>();
      t.offset = rd<uint64_t>();
      uint64_t len;
      if (const char* e = ggml_row_bytes(t.kind, t.dims[0], &len)) throw GgufError(e);
      for (size_t d = 1; d < t.dims.size(); d++) {
        if (len > UINT64_MAX / t.dims[d]) throw GgufError("tensor length overflow");
        len *= t.dims[d];
      }
      t.len = len;
      std::string name = t.name;
      if (!tensors.emplace(std::move(name), std::move(t)).second) throw GgufError("duplicate tensor name");
    }
    uint64_t align = 32;
    auto al = meta.find("general.alignment");
    if (al != meta.end() && !al->second.get_u64(&align)) align = 32;
    if (align == 0 || (align & (align - 1)) || align > 4096) throw GgufError("invalid GGUF alignment");
    const uint64_t start = (at_ + align - 1) & ~(align - 1);
    std::vector<std::pair<uint64_t, uint64_t>> spans;
    for (auto& kv : tensors) {
      GgufTensor& t = kv.second;
      if (t.offset % align) throw GgufError("unaligned tensor " + t.name);
      if (t.offset > UINT64_MAX - start) throw GgufError("tensor offset overflow");
      t.offset += start;
      if (t.len > UINT64_MAX - t.offset) throw GgufError("tensor end overflow");
      if (t.offset + t.len > n_) throw GgufError("truncated tensor " + t.name);
      spans.emplace_back(t.offset, t.offset + t.len);
    }
    std::sort(spans.begin(), spans.end());
    for (size_t k = 1; k < spans.size(); k++)
      if (spans[k - 1].second > spans[k].first) throw GgufError("overlapping tensors");
  }

  const GgufTensor& tensor(const std::string& name) const {
    auto it = tensors.find(name);
    if (it == tensors.end()) throw GgufError("missing tensor " + name);
    return it->second;
  }
  bool has(const std::string& name) const { return tensors.count(name) != 0; }
  bool uint(const std::string& key, uint64_t* out) const {
    auto it = meta.find(key);
    return it != meta.end() && it->second.get_u64(out);
  }
  uint64_t need_uint(const std::string& key) const {
    uint64_t v;
    if (!uint(key, &v)) throw GgufError("missing integer " + key);
    return v;
  }
  float real(const std::string& key, float fallback) const {
    auto it = meta.find(key);
    double v;
    if (it == meta.end() || !it->second.get_f64(&v)) return fallback;
    return (float)v;
  }
  const std::string* str(const std::string& key) const {
    auto it = meta.find(key);
    return it != meta.end() && it->second.type == MetaValue::String ? &it->second.s : nullptr;
  }

 private:
  const uint8_t* p_ = nullptr;
  uint64_t n_ = 0, at_ = 0, budget_ = 0;

  void bytes(void* out, uint64_t k) {
    if (k > n_ - at_) throw GgufError("failed to fill whole buffer");
    memcpy(out, p_ + at_, k);
    at_ += k;
  }
  template <class T>
  T rd() {
    T v;
    bytes(&v, sizeof v);
    return v;
  }
  uint64_t count(uint64_t limit) {
    const uint64_t c = rd<uint64_t>();
    if (c > limit) throw GgufError("GGUF count " + std::to_string(c) + " exceeds limit " + std::to_string(limit));
    return c;
  }
  std::string text() {
    const uint64_t c = count(16ull << 20);
    if (c > budget_) throw GgufError("GGUF metadata budget exceeded");
    budget_ -= c;
    std::string s(c, '\0');
    bytes(&s[0], c);
    return s;
  }
  MetaValue value(uint32_t t, int depth) {
    if (depth > 4 || budget_ < 8) throw GgufError("excessive metadata depth/size");
    budget_ -= 8;
    MetaValue v;
    switch (t) {
      case 0: v.type = MetaValue::Unsigned; v.u = rd<uint8_t>(); break;
      case 1: v.type = MetaValue::Signed; v.i = rd<int8_t>(); break;
      case 2: v.type = MetaValue::Unsigned; v.u = rd<uint16_t>(); break;
      case 3: v.type = MetaValue::Signed; v.i = rd<int16_t>(); break;
      case 4: v.type = MetaValue::Unsigned; v.u = rd<uint32_t>(); break;
      case 5: v.type = MetaValue::Signed; v.i = rd<int32_t>(); break;
      case 6: {
        const float f = rd<float>();
        if (!std::isfinite(f)) throw GgufError("nonfinite metadata");
        v.type = MetaValue::Float;
        v.f = f;
        break;
      }
      case 7: {
        const uint8_t b = rd<uint8_t>();
        if (b > 1) throw GgufError("invalid boolean");
        v.type = MetaValue::Bool;
        v.u = b;
        break;
      }
      case 8: v.type = MetaValue::String; v.s = text(); break;
      case 9: {
        const uint32_t item = rd<uint32_t>();
        const uint64_t c = count(1000000);
        v.type = MetaValue::Array;
        v.n_items = c;
        for (uint64_t k = 0; k < c; k++) value(item, depth + 1);
        break;
      }
      case 10: v.type = MetaValue::Unsigned; v.u = rd<uint64_t>(); break;
      case 11: v.type = MetaValue::Signed; v.i = rd<int64_t>(); break;
      case 12: {
        const double f = rd<double>();
        if (!std::isfinite(f)) throw GgufError("nonfinite metadata");
        v.type = MetaValue::Float;
        v.f = f;
        break;
      }
      default: throw GgufError("unknown GGUF metadata type " + std::to_string(t));
    }
    return v;
  }
};

}  // namespace qc
