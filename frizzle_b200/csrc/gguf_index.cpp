#include "gguf_index.h"

#include <algorithm>
#include <cstring>

namespace fz {
namespace {

// ggml tensor types: block elements and bytes (gguf/types.h's table).
bool block_of(uint32_t type, uint64_t& elements, uint64_t& bytes) {
  switch (type) {
    case 0: elements = 1; bytes = 4; return true;    // F32
    case 1: elements = 1; bytes = 2; return true;    // F16
    case 2: elements = 32; bytes = 18; return true;  // Q4_0
    case 3: elements = 32; bytes = 20; return true;  // Q4_1
    case 8: elements = 32; bytes = 34; return true;  // Q8_0
    default: return false;
  }
}

class Cursor {
 public:
  Cursor(const uint8_t* p, uint64_t n) : p_(p), n_(n) {}
  bool take(void* dst, uint64_t k) {
    if (k > n_ - at_) {
      short_ = at_ + k;
      return false;
    }
    std::memcpy(dst, p_ + at_, k);
    at_ += k;
    return true;
  }
  bool skip(uint64_t k) {
    if (k > n_ - at_) {
      short_ = at_ + k;
      return false;
    }
    at_ += k;
    return true;
  }
  template <typename T>
  bool get(T& v) { return take(&v, sizeof(T)); }
  bool string(std::string& s, uint64_t limit = 1u << 20) {
    uint64_t len = 0;
    if (!get(len)) return false;
    if (len > limit) { bad_ = true; return false; }
    if (len > n_ - at_) { short_ = at_ + len; return false; }
    s.assign(reinterpret_cast<const char*>(p_ + at_), len);
    at_ += len;
    return true;
  }
  uint64_t at() const { return at_; }
  uint64_t needed() const { return short_; }
  bool bad() const { return bad_; }

 private:
  const uint8_t* p_;
  uint64_t n_;
  uint64_t at_ = 0;
  uint64_t short_ = 0;
  bool bad_ = false;
};

uint64_t scalar_size(uint32_t t) {
  switch (t) {
    case 0: case 1: case 7: return 1;
    case 2: case 3: return 2;
    case 4: case 5: case 6: return 4;
    case 10: case 11: case 12: return 8;
    default: return 0;
  }
}

bool read_scalar(Cursor& c, uint32_t t, GgufValue& v) {
  switch (t) {
    case 0: { uint8_t x; if (!c.get(x)) return false; v.u = x; return true; }
    case 1: { int8_t x; if (!c.get(x)) return false; v.i = x; v.u = (uint64_t)x; return true; }
    case 2: { uint16_t x; if (!c.get(x)) return false; v.u = x; return true; }
    case 3: { int16_t x; if (!c.get(x)) return false; v.i = x; v.u = (uint64_t)x; return true; }
    case 4: { uint32_t x; if (!c.get(x)) return false; v.u = x; return true; }
    case 5: { int32_t x; if (!c.get(x)) return false; v.i = x; v.u = (uint64_t)x; return true; }
    case 6: { float x; if (!c.get(x)) return false; v.f = x; return true; }
    case 7: { uint8_t x; if (!c.get(x)) return false; v.u = x; return true; }
    case 10: { uint64_t x; if (!c.get(x)) return false; v.u = x; return true; }
    case 11: { int64_t x; if (!c.get(x)) return false; v.i = x; v.u = (uint64_t)x; return true; }
    case 12: { double x; if (!c.get(x)) return false; v.f = x; return true; }
    default: return false;
  }
}

}  // namespace

const GgufTensor* GgufIndex::find(const std::string& name) const {
  auto it = by_name.find(name);
  return it == by_name.end() ? nullptr : &tensors[it->second];
}

bool GgufIndex::get_u32(const std::string& key, uint32_t& out) const {
  auto it = metadata.find(key);
  if (it == metadata.end()) return false;
  const GgufValue& v = it->second;
  if (v.type == 4 || v.type == 2 || v.type == 0 || v.type == 10) {
    if (v.u > 0xFFFFFFFFull) return false;
    out = (uint32_t)v.u;
    return true;
  }
  if ((v.type == 5 || v.type == 3 || v.type == 1 || v.type == 11) && v.i >= 0 && v.i <= 0xFFFFFFFFll) {
    out = (uint32_t)v.i;
    return true;
  }
  return false;
}

bool GgufIndex::get_f32(const std::string& key, float& out) const {
  auto it = metadata.find(key);
  if (it == metadata.end() || (it->second.type != 6 && it->second.type != 12)) return false;
  out = (float)it->second.f;
  return true;
}

GgufError parse_gguf_index(const uint8_t* bytes, uint64_t n, GgufIndex& out, uint64_t& needed,
                           std::string& message) {
  out = GgufIndex{};
  needed = 0;
  Cursor c(bytes, n);
  auto truncated = [&]() {
    if (c.bad()) {
      message = "a string is longer than the format allows";
      return GgufError::Malformed;
    }
    needed = c.needed();
    message = "the index continues past the bytes given";
    return GgufError::Truncated;
  };
  char magic[4];
  if (!c.take(magic, 4)) return truncated();
  if (std::memcmp(magic, "GGUF", 4) != 0) {
    message = "not a GGUF file (bad magic)";
    return GgufError::BadMagic;
  }
  if (!c.get(out.version)) return truncated();
  if (out.version != 3) {
    message = "GGUF version " + std::to_string(out.version) + " is not 3";
    return GgufError::BadVersion;
  }
  uint64_t tensor_count = 0, kv_count = 0;
  if (!c.get(tensor_count) || !c.get(kv_count)) return truncated();
  if (tensor_count > (1u << 20) || kv_count > (1u << 20)) {
    message = "tensor or metadata count is implausible";
    return GgufError::Malformed;
  }
  for (uint64_t i = 0; i < kv_count; i++) {
    std::string key;
    if (!c.string(key, 1 << 16)) return truncated();
    if (key.empty()) {
      message = "empty metadata key";
      return GgufError::Malformed;
    }
    GgufValue v;
    if (!c.get(v.type)) return truncated();
    if (v.type == 8) {
      if (!c.string(v.s)) return truncated();
    } else if (v.type == 9) {
      if (!c.get(v.array_type) || !c.get(v.array_count)) return truncated();
      if (v.array_type == 9) {
        message = "nested array in " + key;
        return GgufError::Malformed;
      }
      if (v.array_type == 8) {
        for (uint64_t j = 0; j < v.array_count; j++) {
          uint64_t len = 0;
          if (!c.get(len)) return truncated();
          if (len > (1u << 20)) {
            message = "array string too long in " + key;
            return GgufError::Malformed;
          }
          if (!c.skip(len)) return truncated();
        }
      } else {
        const uint64_t sz = scalar_size(v.array_type);
        if (!sz) {
          message = "unknown array value type in " + key;
          return GgufError::Malformed;
        }
        if (v.array_count > (1ull << 40) / sz) {
          message = "array too long in " + key;
          return GgufError::Malformed;
        }
        if (!c.skip(v.array_count * sz)) return truncated();
      }
    } else {
      if (!scalar_size(v.type)) {
        message = "unknown value type in " + key;
        return GgufError::Malformed;
      }
      if (!read_scalar(c, v.type, v)) return truncated();
    }
    if (!out.metadata.emplace(key, v).second) {
      message = "duplicate metadata key " + key;
      return GgufError::Duplicate;
    }
  }
  uint32_t align = 32;
  if (out.metadata.count("general.alignment")) {
    const GgufValue& a = out.metadata["general.alignment"];
    if (a.type != 4 || a.u == 0 || (a.u & (a.u - 1))) {
      message = "general.alignment is not a power-of-two u32";
      return GgufError::Malformed;
    }
    align = (uint32_t)a.u;
  }
  out.alignment = align;
  for (uint64_t i = 0; i < tensor_count; i++) {
    GgufTensor t;
    if (!c.string(t.name, 64)) {
      if (c.bad()) {
        message = "tensor name longer than 64 bytes";
        return GgufError::Malformed;
      }
      return truncated();
    }
    uint32_t nd = 0;
    if (!c.get(nd)) return truncated();
    if (nd == 0 || nd > 4) {
      message = "tensor " + t.name + " has " + std::to_string(nd) + " dimensions";
      return GgufError::Malformed;
    }
    t.elements = 1;
    for (uint32_t d = 0; d < nd; d++) {
      uint64_t dim = 0;
      if (!c.get(dim)) return truncated();
      if (dim == 0 || dim > (1ull << 40) || t.elements > (1ull << 48) / dim) {
        message = "tensor " + t.name + " has an invalid dimension";
        return GgufError::Malformed;
      }
      t.dims.push_back(dim);
      t.elements *= dim;
    }
    if (!c.get(t.type) || !c.get(t.offset)) return truncated();
    uint64_t be = 0, bb = 0;
    if (!block_of(t.type, be, bb)) {
      message = "tensor " + t.name + " has unknown type " + std::to_string(t.type);
      return GgufError::Malformed;
    }
    if (t.dims[0] % be) {
      message = "tensor " + t.name + " rows are not whole blocks";
      return GgufError::Malformed;
    }
    if (t.offset % align) {
      message = "tensor " + t.name + " offset is not aligned";
      return GgufError::Malformed;
    }
    t.bytes = t.elements / be * bb;
    // The offset comes from the file: its end must not wrap past 2^64, or
    // every later bound (data in the file, no overlap) would pass on the
    // wrapped value.
    if (t.offset > UINT64_MAX - t.bytes) {
      message = "tensor " + t.name + " offset is out of range";
      return GgufError::Malformed;
    }
    if (out.by_name.count(t.name)) {
      message = "duplicate tensor " + t.name;
      return GgufError::Duplicate;
    }
    out.by_name[t.name] = out.tensors.size();
    out.tensors.push_back(std::move(t));
  }
  out.data_offset = (c.at() + align - 1) / align * align;
  // Tensors may not overlap one another.
  std::vector<std::pair<uint64_t, uint64_t>> spans;
  for (const GgufTensor& t : out.tensors) spans.push_back({t.offset, t.offset + t.bytes});
  std::sort(spans.begin(), spans.end());
  for (size_t i = 1; i < spans.size(); i++)
    if (spans[i].first < spans[i - 1].second) {
      message = "tensor data overlaps";
      return GgufError::Malformed;
    }
  return GgufError::Ok;
}

}  // namespace fz
