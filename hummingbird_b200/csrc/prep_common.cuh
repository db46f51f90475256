// Helpers for the prologue kernels that turn the raw `to_qkv` projection into prepared attention tiles.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>

#include "attn_internal.h"
#include "hb_sm100.cuh"

namespace hb {

// 8 bf16 of one 16-byte chunk <-> fp32
__device__ __forceinline__ void unpack8(const uint4& v, float (&x)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[2 * i] = bf16_lo(w[i]);
    x[2 * i + 1] = bf16_hi(w[i]);
  }
}
__device__ __forceinline__ uint4 pack8(const float (&x)[8]) {
  return make_uint4(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]), pack_bf16x2(x[4], x[5]),
                    pack_bf16x2(x[6], x[7]));
}

// 128-bit read-only load that bypasses L1 allocation (each chunk is read once by the prologue)
__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// Partner 16-byte chunk for the half-half rotate of a 64-dim head split into eight 8-dim chunks:
// dims [0, half) pair with d + half, the rest with d - half (band_attention.py:77, 84).
__device__ __forceinline__ int rope_partner_chunk(int c, int hc8) { return c < hc8 ? c + hc8 : c - hc8; }

// 2 pi = kTwoPi1 + kTwoPi2 + kTwoPi3 (fp32 parts of 2 pi taken to 60 digits) and fp32(1 / (2 pi))
constexpr float kTwoPi1 = 6.2831854820251465f, kTwoPi2 = -1.7484555314695172e-07f, kTwoPi3 = -6.8604980400235275e-15f;
constexpr float kInvTwoPi = 0.15915493667125702f;

// cos / sin of an fp32 angle: Cody-Waite reduction by 2 pi (three-part constant, FMA) to |r| <= ~pi, then
// the hardware approximations on the reduced argument (absolute error ~2^-21 there).
__device__ __forceinline__ void sincos_reduced(float x, float& sn, float& cs) {
  // k = rint(x / 2 pi) by adding and subtracting 1.5 * 2^23 (exact for |x / 2 pi| < 2^22), on the FMA pipe
  const float k = __fadd_rn(__fmaf_rn(x, kInvTwoPi, 12582912.0f), -12582912.0f);
  float r = fmaf(-k, kTwoPi1, x);
  r = fmaf(-k, kTwoPi2, r);
  r = fmaf(-k, kTwoPi3, r);
  sn = __sinf(r);
  cs = __cosf(r);
}

}  // namespace hb
