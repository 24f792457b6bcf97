// C entry points over the reference's own edit and prefix code, compiled in
// place from the plainsight-systems/frizzle sources (src/core/edit/edit.cpp,
// src/core/cache/prefix.cpp).  TEST INFRASTRUCTURE ONLY: it pins the oracle's
// and the engine's edit-table handling to the reference itself.  Built by
// `make ref` into oracle/_ref/, never committed, and only when the reference
// sources are present.
#include <cstdint>
#include <cstring>
#include <span>
#include <vector>

#include "core/cache/prefix.h"
#include "core/edit/edit.h"

namespace {
struct RefEdit {
  std::uint32_t layer, neuron, kind;
  float value;
  std::uint32_t from, until;
};

std::vector<frizzle::edit::Edit> edits_of(const RefEdit* in, std::size_t n) {
  std::vector<frizzle::edit::Edit> out;
  out.reserve(n);
  for (std::size_t i = 0; i < n; ++i) {
    out.push_back({in[i].layer, in[i].neuron, static_cast<frizzle::edit::EditKind>(in[i].kind), in[i].value,
                   in[i].from, in[i].until});
  }
  return out;
}

frizzle::model::ModelDescription model_of(std::uint32_t layers, std::uint32_t width) {
  frizzle::model::ModelDescription m{};
  frizzle::model::LayerDescription l{};
  l.feed_forward_width = width;
  m.layers.assign(layers, l);
  return m;
}
}  // namespace

extern "C" {
int ref_edit_check(const RefEdit* edits, std::size_t n, std::uint32_t layers, std::uint32_t width,
                   std::size_t* index, char* subject, std::size_t cap) {
  const auto e = edits_of(edits, n);
  const auto r = frizzle::edit::check(e, model_of(layers, width));
  *index = r.index;
  if (cap) {
    std::strncpy(subject, r.subject.c_str(), cap - 1);
    subject[cap - 1] = 0;
  }
  return static_cast<int>(r.error);
}

std::size_t ref_edit_table(const RefEdit* edits, std::size_t n, std::uint32_t layers, std::uint32_t width,
                           std::uint32_t origin, std::uint32_t* out, std::size_t cap) {
  const auto words = frizzle::edit::table(edits_of(edits, n), model_of(layers, width), origin);
  if (words.size() <= cap) std::memcpy(out, words.data(), words.size() * 4);
  return words.size();
}

float ref_edit_apply(std::uint32_t kind, float value, float neuron) {
  return frizzle::edit::apply(static_cast<frizzle::edit::EditKind>(kind), value, neuron);
}

std::uint32_t ref_first_edit_difference(const RefEdit* a, std::size_t na, const RefEdit* b, std::size_t nb) {
  return frizzle::cache::first_edit_difference(edits_of(a, na), edits_of(b, nb));
}

std::size_t ref_longest_common_prefix(const std::uint32_t* a, std::size_t na, const std::uint32_t* b,
                                      std::size_t nb) {
  std::vector<frizzle::tokenizer::TokenId> x(na), y(nb);
  for (std::size_t i = 0; i < na; ++i) x[i] = static_cast<frizzle::tokenizer::TokenId>(a[i]);
  for (std::size_t i = 0; i < nb; ++i) y[i] = static_cast<frizzle::tokenizer::TokenId>(b[i]);
  return frizzle::cache::longest_common_prefix(x, y);
}
}
