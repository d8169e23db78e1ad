// Shared definitions of the decode-MoE path: the routing plan written by the
// router kernel and read by the gate|up and down kernels, and the scratch layout.
#pragma once

#include <stddef.h>
#include <stdint.h>

namespace duplex {

constexpr int kMaxTokens = 8;    // mma N: tokens that share one pass over an expert
constexpr int kMaxTopK = 8;
constexpr int kMaxExperts = 256;
constexpr int kMaxUnits = kMaxTokens * kMaxTopK;  // distinct experts touched by <= 8 tokens

// One "unit" is a distinct expert selected by at least one of the T tokens.  Its
// weights are streamed once; batch column n of the MMA carries token n.
struct MoePlan {
  int n_units;
  int pad_[3];
  int unit_expert[kMaxUnits];
  uint32_t unit_mask[kMaxUnits];          // bit n: token n selected this expert
  float unit_w[kMaxUnits * kMaxTokens];   // routing weight of (unit, token), 0 if unselected
};

// Scratch layout inside the caller's workspace (all offsets 256-byte aligned).
struct MoeScratch {
  size_t counter, logits, plan, w, sel, xn, act, total;
};

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

inline MoeScratch moe_scratch_layout(int T, int E, int H, int I, int top_k) {
  MoeScratch s;
  size_t off = 0;
  s.counter = off; off += 256;
  s.logits = off; off += align_up((size_t)T * E * 4, 256);
  s.plan = off; off += align_up(sizeof(MoePlan), 256);
  s.w = off; off += align_up((size_t)T * top_k * 4, 256);
  s.sel = off; off += align_up((size_t)T * top_k * 4, 256);
  s.xn = off; off += align_up((size_t)T * H * 2, 256);     // RMS-normalised tokens
  int units = T * top_k < E ? T * top_k : E;
  if (units > kMaxUnits) units = kMaxUnits;
  s.act = off; off += align_up((size_t)units * kMaxTokens * I * 2, 256);
  s.total = off;
  return s;
}

}  // namespace duplex
