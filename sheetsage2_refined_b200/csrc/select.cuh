// Greedy selection keys shared by every path that picks a token.
//
// The reference picks `logits.masked_fill(~allowed, -inf).argmax(-1)`
// (engine.py:349-350): the largest value, the lowest index among equal
// values, and index 0 for a row whose best value is -inf (every token masked,
// or every allowed value pushed to -inf by a bias).  torch.argmax compares
// values, so -0.0 and +0.0 tie, and a NaN counts as larger than any number.
//
// A key packs an order-preserving image of the value in its high word and
// ~index in its low word, so that the 64-bit maximum over (value, index)
// pairs is the reference's choice and can be formed with atomicMax across
// CTAs in any order.  A key of 0 means "nothing allowed" (no real key is 0).
#pragma once

#include <stdint.h>

namespace s2r {

// Row m's key lives at keys[m * kKeyStride]: one 128-byte line per row, so
// that the atomics of different rows go to different L2 lines.
constexpr int kKeyStride = 16;

__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
  uint32_t u = __float_as_uint(v);
  if (u == 0x80000000u) u = 0u;        // -0 ties with +0
  if (v != v) u = 0x7fffffffu;         // every NaN ranks above +inf, ties among NaNs go to the lowest index
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (unsigned long long)(0xffffffffu - (uint32_t)idx);
}

// The token of a row's maximum key: its index, or 0 when the best value is
// -inf or nothing was allowed.  The image of -inf is ~0xff800000 = 0x007fffff;
// every larger value has a larger image.
__device__ __forceinline__ int64_t key_token(unsigned long long k) {
  return (k >> 32) > 0x007fffffull ? (int64_t)(0xffffffffu - (uint32_t)(k & 0xffffffffull)) : 0;
}

}  // namespace s2r
