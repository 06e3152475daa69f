// requant.cuh - TFLite per-channel requantisation on the device.
//
// Follows TFLite's MultiplyByQuantizedMultiplier (double-rounding form):
//   x' = x << max(shift, 0)                    (wrapping, as in int32)
//   h  = SaturatingRoundingDoublingHighMul(x', M)   gemmlowp
//   r  = RoundingDivideByPOT(h, max(-shift, 0))      gemmlowp
// then out = clamp(r + zp_out, act_min, act_max).
//
// gemmlowp computes h as (x'*M + nudge) / 2^31 truncated toward zero, with
// nudge = 2^30 for a non-negative product and 1 - 2^30 otherwise.  For a
// product p < 0 that is ceil((p + 1 - 2^30) / 2^31) = floor((p + 2^30) / 2^31),
// and for p >= 0 it is floor((p + 2^30) / 2^31) directly, so in both cases
// h = (p + 2^30) >> 31 with an arithmetic shift.  Only x' = M = INT32_MIN
// saturates, which a non-negative TFLite multiplier never produces; it is
// still handled.
#pragma once

#include <cstdint>

namespace pspml {

__device__ __forceinline__ int32_t mbqm_dev(int32_t x, int32_t m, int32_t shift) {
  const int32_t left = shift > 0 ? shift : 0;
  const int32_t right = shift > 0 ? 0 : -shift;
  const int32_t a = static_cast<int32_t>(static_cast<uint32_t>(x) << left);
  int32_t h = static_cast<int32_t>((static_cast<int64_t>(a) * m + (1ll << 30)) >> 31);
  if (a == INT32_MIN && m == INT32_MIN) h = INT32_MAX;
  const int32_t mask = static_cast<int32_t>((1u << right) - 1u);
  const int32_t rem = h & mask;
  const int32_t thr = (mask >> 1) + (h < 0 ? 1 : 0);
  return (h >> right) + (rem > thr ? 1 : 0);
}

struct ActParams {
  int32_t zp_out, act_min, act_max;
};

__device__ __forceinline__ int32_t finish_dev(int32_t acc, int32_t m, int32_t shift,
                                              const ActParams& ap) {
  int32_t v = mbqm_dev(acc, m, shift) + ap.zp_out;
  v = v < ap.act_min ? ap.act_min : v;
  v = v > ap.act_max ? ap.act_max : v;
  return v;
}

__device__ __forceinline__ uint32_t pack4_s8(int32_t a, int32_t b, int32_t c, int32_t d) {
  return (static_cast<uint32_t>(a) & 0xFFu) | ((static_cast<uint32_t>(b) & 0xFFu) << 8) |
         ((static_cast<uint32_t>(c) & 0xFFu) << 16) | ((static_cast<uint32_t>(d) & 0xFFu) << 24);
}

__device__ __forceinline__ int32_t sbyte(uint32_t w, int i) {
  return static_cast<int32_t>(static_cast<int8_t>((w >> (8 * i)) & 0xFFu));
}

}  // namespace pspml
