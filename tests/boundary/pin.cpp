// Compile-time pin of the C ABI's step and record structs to the reference's
// own definitions: kernels::Step's 64-byte head
// (src/core/kernels/interface.h:163-185) and sampler::SampledRecord
// (src/core/sampler/sampler.h:187-193).  Test infrastructure: compiled by
// tests/test_boundary.py with g++ -std=c++23 against the reference checkout.
#include <cstddef>

#include "core/kernels/interface.h"
#include "core/sampler/sampler.h"
#include "frizzle_b200.h"

using frizzle::kernels::kStepHead;
using frizzle::kernels::Step;
using frizzle::sampler::SampledRecord;

#define SAME_FIELD(ours, theirs)                                                       \
  static_assert(offsetof(fz_step, ours) == offsetof(Step, theirs), #ours " offset"); \
  static_assert(sizeof(fz_step::ours) == sizeof(Step::theirs), #ours " size")

SAME_FIELD(position, position);
SAME_FIELD(tokens, tokens);
SAME_FIELD(logits, logits);
SAME_FIELD(fed, fed);
SAME_FIELD(seed, seed);
SAME_FIELD(top_k, top_k);
SAME_FIELD(temperature, temperature);
SAME_FIELD(top_p, top_p);
SAME_FIELD(min_p, min_p);
SAME_FIELD(log_min_p, log_min_p);
// `capture` and the padding fill the reference's padding words, which end
// where its identifiers begin.
static_assert(offsetof(fz_step, capture) == offsetof(Step, padding), "capture takes the first padding word");
static_assert(offsetof(fz_step, padding) + sizeof(fz_step::padding) == offsetof(Step, ids), "head ends at ids");
static_assert(sizeof(fz_step) == kStepHead, "fz_step is the 64-byte step head");

static_assert(sizeof(fz_record) == sizeof(SampledRecord), "record size");
static_assert(offsetof(fz_record, token) == offsetof(SampledRecord, token), "token");
static_assert(offsetof(fz_record, failed) == offsetof(SampledRecord, failed), "failed");
static_assert(offsetof(fz_record, u) == offsetof(SampledRecord, u), "u");
static_assert(offsetof(fz_record, padding) == offsetof(SampledRecord, padding), "padding");

int main() { return 0; }
