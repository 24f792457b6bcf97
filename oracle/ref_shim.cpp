// C entry points over the reference's own edit, prefix, KV-cache bookkeeping
// and capture-layout code, compiled in place from the
// plainsight-systems/frizzle sources (src/core/edit/edit.cpp,
// src/core/cache/prefix.cpp, src/core/cache/kv.cpp,
// src/core/capture/capture.cpp).  TEST INFRASTRUCTURE ONLY: it pins the
// oracle's and the engine's edit-table handling and capture-store layout to
// the reference itself.  Built by
// `make ref` into oracle/_ref/, never committed, and only when the reference
// sources are present.
#include <cstdint>
#include <cstring>
#include <span>
#include <vector>

#include "core/cache/kv.h"
#include "core/cache/prefix.h"
#include "core/capture/capture.h"
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

// capture::layout() of a Gemma-3-shaped description: `layers` layers of
// `width` embedding, `ffn` feed-forward, `heads` query heads of `head_dim`,
// window `window` except every `pattern`-th layer (pattern - 1, 2 pattern - 1,
// ...), which attends over the trained context `context`.  Per layer 20 words
// into out: the eight slots' (first, width) in capture.h's order, then keys,
// query heads, window and full attention.  Returns the store's words.
std::uint64_t ref_capture_layout(std::uint32_t layers, std::uint32_t width, std::uint32_t ffn,
                                 std::uint32_t heads, std::uint32_t head_dim, std::uint32_t window,
                                 std::uint32_t pattern, std::uint32_t context, std::uint32_t* out) {
  frizzle::model::ModelDescription m{};
  m.embedding_width = width;
  m.trained_context = context;
  m.layers.resize(layers);
  for (std::uint32_t l = 0; l < layers; ++l) {
    auto& d = m.layers[l];
    d.query_heads = heads;
    d.key_value_heads = 1;
    d.head_dimension = head_dim;
    d.feed_forward_width = ffn;
    d.attention_window = l % pattern == pattern - 1 ? context : window;
  }
  const auto lay = frizzle::capture::layout(m);
  for (std::uint32_t l = 0; l < layers; ++l) {
    const auto& s = lay.layers[l];
    const frizzle::capture::Slot slots[8] = {s.neurons, s.residual, s.attention_added, s.mlp_added,
                                             s.query,   s.weights,  s.stats,           s.readout};
    std::uint32_t* o = out + 20 * l;
    for (int i = 0; i < 8; ++i) {
      o[2 * i] = slots[i].first;
      o[2 * i + 1] = slots[i].width;
    }
    o[16] = s.keys;
    o[17] = s.query_heads;
    o[18] = s.window;
    o[19] = s.full_attention ? 1u : 0u;
  }
  return lay.words;
}

// A KvCache over `layers` layers of the given windows and ring slots, run
// through n operations: op[2i] 0 = advance(op[2i + 1]), 1 =
// truncate(op[2i + 1]).  After operation i, out[2i] is its result (truncate's
// return, or the new length after an advance) and out[2i + 1] the length.
void ref_kv_run(const std::uint32_t* windows, const std::uint32_t* slots, std::uint32_t layers,
                std::uint32_t capacity, const std::uint32_t* op, std::size_t n, std::uint32_t* out) {
  frizzle::model::ModelDescription m{};
  m.layers.resize(layers);
  frizzle::residency::ResidencyPlan plan{};
  plan.cache.resize(layers);
  for (std::uint32_t l = 0; l < layers; ++l) {
    m.layers[l].attention_window = windows[l];
    plan.cache[l].slots = slots[l];
  }
  frizzle::cache::KvCache kv(m, plan, frizzle::policy::CachePrecision{}, capacity);
  for (std::size_t i = 0; i < n; ++i) {
    if (op[2 * i] == 0) {
      kv.advance(op[2 * i + 1]);
      out[2 * i] = kv.length();
    } else {
      out[2 * i] = kv.truncate(op[2 * i + 1]);
    }
    out[2 * i + 1] = kv.length();
  }
}

std::size_t ref_longest_common_prefix(const std::uint32_t* a, std::size_t na, const std::uint32_t* b,
                                      std::size_t nb) {
  std::vector<frizzle::tokenizer::TokenId> x(na), y(nb);
  for (std::size_t i = 0; i < na; ++i) x[i] = static_cast<frizzle::tokenizer::TokenId>(a[i]);
  for (std::size_t i = 0; i < nb; ++i) y[i] = static_cast<frizzle::tokenizer::TokenId>(b[i]);
  return frizzle::cache::longest_common_prefix(x, y);
}
}
