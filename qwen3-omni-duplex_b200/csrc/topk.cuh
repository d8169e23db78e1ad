// Order keys of router logits for the top-k (persistent stack and grouped MoE).
#pragma once

#include "common.cuh"

namespace duplex {

// Logits are rounded to the 16-bit activation type, so (ordered 16-bit value << 15)
// | (0x7FFF - expert) is a unique 31-bit key per expert and "k > v" is the sign of
// v - k: larger logit first, ties to the lower expert id, NaN above everything (as
// torch.topk), -0 equal to +0.  Every CTA derives the same selection from the same
// logits, whatever their values.  Never 0 for a real logit.
template <typename T>
DEVI uint32_t order_key(float f, int e) {
  const T h = from_f32<T>(f);
  uint32_t b = (uint32_t)*reinterpret_cast<const uint16_t*>(&h);
  const bool nan = DqOff<T>::kOddDiv16 ? ((b & 0x7C00u) == 0x7C00u && (b & 0x3FFu))
                                       : ((b & 0x7F80u) == 0x7F80u && (b & 0x7Fu));
  if (b == 0x8000u) b = 0u;
  b = nan ? 0xFFFFu : ((b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u));
  return (b << 15) | (0x7FFFu - (uint32_t)e);
}

DEVI int key_expert(uint32_t key) { return (int)(0x7FFFu - (key & 0x7FFFu)); }

}  // namespace duplex
