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

// Per-channel requantisation constants (16 bytes, one vector load).
//
// Fast form, for a right shift r = -shift in [1, 23] (every calibrated TFLite
// layer): with a = acc + bias, p = a * M and C = 2^30 + 2^(30+r) + zp * 2^(31+r),
//   out + zp_out = floor((p + C - [a < 0] * 2^31) / 2^(31 + r))
// which equals RoundingDivideByPOT(SaturatingRoundingDoublingHighMul(a, M), r)
// + zp_out exactly: the high-mul rounding is floor((p + 2^30) / 2^31); the
// POT division adds 2^(r-1) minus one for a negative high-mul result and
// floors; floor((floor(x / A) + k) / B) = floor((x + k*A) / (A*B)) merges the
// two floors; and replacing [high-mul < 0] by [a < 0] only differs when the
// high-mul is 0, where both give 0 for r >= 1.  With t = p + C split into
// 32-bit halves (lo, hi), the [a < 0] * 2^31 correction lowers hi by one
// exactly when a < 0 and lo < 2^31, so
//   out + zp_out = (hi + ((a & ~lo) >> 31)) >> (r - 1).
// |p| < 2^62 and |C| < 2^62 for r <= 23, so t never overflows.
// The table stores C - 2^32 (one less in the high word); with t' = p + C - 2^32
// the same result is (hi' + ((~a | lo) >>> 31)) >> (r - 1), because
// 1 - ([a < 0] & ~lo[31]) = (~a | lo)[31]: one LOP3 and one shifted add.
// Other shifts (left shifts, r == 0, r > 23) take the general path: sr < 0,
// c_lo holds the TFLite shift and c_hi the output zero point.
struct __align__(16) RqChannel {
  int32_t m;
  uint32_t c_lo;
  int32_t c_hi;
  int32_t sr;
};

__host__ __device__ inline RqChannel make_rq(int32_t m, int32_t shift, int32_t zp_out) {
  RqChannel q;
  const int32_t r = -shift;
  if (m > 0 && r >= 1 && r <= 23) {
    const int64_t c = (int64_t{1} << 30) + (int64_t{1} << (30 + r)) +
                      static_cast<int64_t>(zp_out) * (int64_t{1} << (31 + r)) -
                      (int64_t{1} << 32);
    q.m = m;
    q.c_lo = static_cast<uint32_t>(static_cast<uint64_t>(c));
    q.c_hi = static_cast<int32_t>(c >> 32);
    q.sr = r - 1;
  } else {
    q.m = m;
    q.c_lo = static_cast<uint32_t>(shift);
    q.c_hi = zp_out;
    q.sr = -1;
  }
  return q;
}

// requantised value + zp_out, before clamping: fast form only (q.sr >= 0).
__device__ __forceinline__ int32_t rq_fast(int32_t a, const RqChannel& q) {
  const int64_t c =
      static_cast<int64_t>((static_cast<uint64_t>(static_cast<uint32_t>(q.c_hi)) << 32) | q.c_lo);
  const int64_t t = static_cast<int64_t>(a) * q.m + c;
  const uint32_t lo = static_cast<uint32_t>(t);
  const int32_t hi = static_cast<int32_t>(t >> 32);
  return (hi + static_cast<int32_t>((~static_cast<uint32_t>(a) | lo) >> 31)) >> q.sr;
}

// Floor form, for ops whose activation clamp starts at or above the output
// zero point (act_min >= zp_out: ReLU, ReLU6, ...): the [a < 0] correction
// of the fast form is left out,
//   out + zp_out = floor((p + C) / 2^(31 + r)) = (hi' + 1) >> (r - 1)
// with hi' the high word of p + (C - 2^32) as the table stores it.  For
// a >= 0 the correction is zero, so this is the fast form.  For a < 0 (so
// p <= -M < 0) both this value and TFLite's are at most zp_out: TFLite's
// high-mul and power-of-two division keep the sign of a, and here
// p + 2^30 + 2^(30+r) < 2^(31+r).  After the clamp to [act_min, act_max]
// both are act_min.  Two instructions fewer than the fast form.
__device__ __forceinline__ int32_t rq_fast_floor(int32_t a, const RqChannel& q) {
  const int64_t c =
      static_cast<int64_t>((static_cast<uint64_t>(static_cast<uint32_t>(q.c_hi)) << 32) | q.c_lo);
  const int64_t t = static_cast<int64_t>(a) * q.m + c;
  return (static_cast<int32_t>(t >> 32) + 1) >> q.sr;
}

// Floor form with the bias folded in: for an accumulator `acc` whose bias is
// `bias`, (acc + bias) * M + C + 2^32 = acc * M + D with D returned here, so
// rq_floor_folded(acc, q.m, D, q.sr) == rq_fast_floor(acc + bias, q) for
// every int32 acc (the same 64-bit integer, formed in another order).
__device__ __forceinline__ int64_t floor_addend(int32_t bias, const RqChannel& q) {
  const int64_t c =
      static_cast<int64_t>((static_cast<uint64_t>(static_cast<uint32_t>(q.c_hi)) << 32) | q.c_lo);
  return static_cast<int64_t>(bias) * q.m + c + (int64_t{1} << 32);
}
__device__ __forceinline__ int32_t rq_floor_folded(int32_t acc, int32_t m, int64_t d,
                                                   int32_t sr) {
  return static_cast<int32_t>((static_cast<int64_t>(acc) * m + d) >> 32) >> sr;
}

// requantised value + zp_out, before clamping; any channel.
__device__ __forceinline__ int32_t rq_apply(int32_t a, const RqChannel& q) {
  if (q.sr >= 0) return rq_fast(a, q);
  return mbqm_dev(a, q.m, static_cast<int32_t>(q.c_lo)) + q.c_hi;
}

// Requantisation forms a kernel is compiled for.
constexpr int kRqGeneral = 0;  // any channel: closed form or the literal steps
constexpr int kRqFast = 1;     // every channel of the op has a fast-form entry
constexpr int kRqFloor = 2;    // fast form and act_min >= zp_out (rq_fast_floor)

// Requantisation selected at compile time.
template <int RQ>
__device__ __forceinline__ int32_t rq_sel(int32_t a, const RqChannel& q) {
  if constexpr (RQ == kRqFloor) return rq_fast_floor(a, q);
  if constexpr (RQ == kRqFast) return rq_fast(a, q);
  return rq_apply(a, q);
}

// The form of an op: `all_fast` when every channel has a fast-form entry.
inline int rq_form(bool all_fast, int32_t act_min, int32_t zp_out) {
  if (!all_fast) return kRqGeneral;
  return act_min >= zp_out ? kRqFloor : kRqFast;
}

__device__ __forceinline__ RqChannel load_rq(const RqChannel* p) {
  const int4 v = __ldg(reinterpret_cast<const int4*>(p));
  RqChannel q;
  q.m = v.x;
  q.c_lo = static_cast<uint32_t>(v.y);
  q.c_hi = v.z;
  q.sr = v.w;
  return q;
}

// Four int32 -> four int8 with saturation to [-128, 127], x0 in byte 0.
// cvt.pack.sat.s8.s32.b32 d, a, b, c gives d = (c << 16) | sat(a) << 8 | sat(b).
__device__ __forceinline__ uint32_t pack_sat4(int32_t x0, int32_t x1, int32_t x2, int32_t x3) {
  uint32_t hi, d;
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, 0;" : "=r"(hi) : "r"(x3), "r"(x2));
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(x1), "r"(x0), "r"(hi));
  return d;
}

// Clamp of four packed int8 lanes to [lo, hi] (bytes replicated).
__device__ __forceinline__ uint32_t clamp4(uint32_t v, uint32_t lo4, uint32_t hi4) {
  return __vmins4(__vmaxs4(v, lo4), hi4);
}

__host__ __device__ inline uint32_t splat4(int32_t v) {
  return (static_cast<uint32_t>(v) & 0xFFu) * 0x01010101u;
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
