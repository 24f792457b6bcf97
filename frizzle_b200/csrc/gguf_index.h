// GGUF v3 index: header, metadata and tensor infos, parsed from the file's
// first bytes with every length and offset checked against what was given
// (the contract of Frizzle's reader, src/core/gguf/reader.h:185 and
// src/core/gguf/types.h:136-166).  Only what the engine reads is kept.
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace fz {

enum class GgufError {
  Ok,
  Truncated,     // more bytes are needed: `needed` says how many
  BadMagic,
  BadVersion,
  Malformed,     // a length, type or count outside what the format allows
  Duplicate,
};

struct GgufValue {
  uint32_t type = 0;
  uint64_t u = 0;     // unsigned and boolean scalars
  int64_t i = 0;      // signed scalars
  double f = 0.0;     // floats
  std::string s;      // strings
  uint32_t array_type = 0;
  uint64_t array_count = 0;
};

struct GgufTensor {
  std::string name;
  std::vector<uint64_t> dims;   // innermost first
  uint32_t type = 0;
  uint64_t offset = 0;          // relative to the data section
  uint64_t elements = 0;
  uint64_t bytes = 0;
};

struct GgufIndex {
  uint32_t version = 0;
  std::map<std::string, GgufValue> metadata;
  std::vector<GgufTensor> tensors;
  std::map<std::string, size_t> by_name;
  uint64_t alignment = 32;
  uint64_t data_offset = 0;     // absolute

  const GgufTensor* find(const std::string& name) const;
  bool get_u32(const std::string& key, uint32_t& out) const;
  bool get_f32(const std::string& key, float& out) const;
};

// Parses `bytes[0, n)`.  On Truncated, `needed` is a byte count that would let
// parsing progress further.  `message` names what was refused.
GgufError parse_gguf_index(const uint8_t* bytes, uint64_t n, GgufIndex& out, uint64_t& needed,
                           std::string& message);

}  // namespace fz
