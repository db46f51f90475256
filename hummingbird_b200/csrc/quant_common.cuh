// Per-row int8 quantisation arithmetic shared by the standalone quantiser (w8a8.cu) and the GLU's fused
// quantisation (dit_glue.cu): q = clamp(rint(x / s), -127, 127) with x / s the correctly rounded fp32 quotient,
// computed without a division per element.
#pragma once
#include <cstdint>

namespace hb {

// rintf(x / s) from q0 = x * fl(1 / s). q0 is within 2^-23 |x / s| of the exact quotient and fl(x / s) within
// 2^-24 |x / s|, so for |q0| < 128.5 the two differ by less than 2^-15: unless q0 lies within 2^-14 of a
// half-integer, fl(x / s) rounds to the same integer n as q0. Quotients of magnitude 128.5 and above clamp to
// +-127 either way. Near-ties and a q0 that is not finite (a reciprocal that overflowed) take the IEEE division.
// n is rounded by adding and subtracting kRoundMagic = 1.5 * 2^23: for |v| < 2^22 the sum lies in [2^23, 2^24),
// where the fp32 spacing is 1, so fl(v + kRoundMagic) - kRoundMagic is v rounded to the nearest integer, ties
// to even (kRoundMagic is even), as rintf gives; larger |v| keep their sign and a magnitude far above 127.
// These are adds on the FMA pipe in place of a division, or of rounding and conversion instructions on the
// transcendental pipe, which the GLU's exponentials and reciprocals already saturate.
constexpr float kRoundMagic = 12582912.f;
constexpr float kNearHalf = 0.5f - 0x1p-14f;

__device__ __forceinline__ float rint_quotient(float x, float s, float rs) {
  const float q0 = x * rs;
  const float n = __fsub_rn(__fadd_rn(q0, kRoundMagic), kRoundMagic);
  if (!(fabsf(q0 - n) < kNearHalf)) return rintf(__fdiv_rn(x, s));
  return n;
}

// clamp(rint(x / s), -127, 127) as a float; rs = __frcp_rn(s).
__device__ __forceinline__ float quantize_int8(float x, float s, float rs) {
  return fminf(fmaxf(rint_quotient(x, s, rs), -127.f), 127.f);
}

// The low byte (two's complement) of an integer-valued v in [-127, 127]: v + kRoundMagic is exact and its bit
// pattern is that of kRoundMagic (low byte 0) plus v.
__device__ __forceinline__ uint32_t int8_bits(float v) { return __float_as_uint(__fadd_rn(v, kRoundMagic)) & 0xFFu; }

}  // namespace hb
