// quant_core.cuh — the element arithmetic of the per-row int8 quantiser, shared
// by the plain quantiser (quantize.cu) and the fused producers (fused.cu).
//
// Contract: s = RN(amax / 127) (1 for an all-zero row), q = clamp(rint(RN(x / s)),
// -127, 127), rint = round half to even.
//
// Fast form, 3 fused fp32 instructions + 1 compare per element, no conversion
// unit. With p = x * inv_s taken exactly (inv_s = RN(1 / s)):
//   t = RN(p + 1.5 * 2^23)       = 1.5 * 2^23 + rint(p) (|p| < 2^22: the sum has
//                                  an ulp of 1, and 1.5 * 2^23 is even)
//   r = t - 1.5 * 2^23           (exact) = rint(p)
//   d = RN(p - r)                (one rounding of the exact distance)
// and the low byte of t's bit pattern is rint(p) mod 256 (1.5 * 2^23 is a
// multiple of 256 in its integer mantissa), i.e. the two's-complement int8.
//
// Why it equals the contract: for a normal s, |p - x/s| <= 2^-24 |x/s| and
// |RN(x/s) - x/s| <= 2^-24 |x/s|, with |x/s| <= 127.0001, so p and the correctly
// rounded quotient RN(x / s) are within 1.6e-5 of each other. Whenever
// |d| <= 0.4999 (p at least 1e-4 away from every half-integer) both round to
// the same integer, and |p| <= 127.0001 makes the clamp a no-op. Every other
// element — near a tie, NaN (the comparison fails), or a row whose scale is
// subnormal or infinite (inv_s passed as 0) — is redone with the exact IEEE
// division and the explicit clamp, four elements at a time. About 1e-3 of
// 4-element groups take that path.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace lema {

constexpr float kRoundMagic = 12582912.0f;  // 1.5 * 2^23
constexpr float kTieGuard = 0.4999f;

__device__ __forceinline__ float quant_row_scale(float amax) {
  return amax > 0.f ? __fdiv_rn(amax, 127.f) : 1.f;
}

// RN(1 / s) for a normal finite scale, else 0 (every element then takes the
// exact division).
__device__ __forceinline__ float quant_row_inv_scale(float s) {
  return (s >= 1.17549435e-38f && s <= 3.40282347e38f) ? __frcp_rn(s) : 0.f;
}

// The contract for one element, by exact division.
__device__ __forceinline__ int32_t quant_exact(float x, float s) {
  int q = __float2int_rn(__fdiv_rn(x, s));
  return max(-127, min(127, q));
}

__device__ __forceinline__ uint32_t pack4_low_bytes(uint32_t a, uint32_t b, uint32_t c,
                                                    uint32_t d) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// The exact path for 4 values. Kept out of line: inlined, the compiler
// if-converts it and the divisions run for every element.
static __device__ __noinline__ uint32_t quant4_exact(float x0, float x1, float x2, float x3, float s) {
  return pack4_low_bytes(static_cast<uint32_t>(quant_exact(x0, s)),
                         static_cast<uint32_t>(quant_exact(x1, s)),
                         static_cast<uint32_t>(quant_exact(x2, s)),
                         static_cast<uint32_t>(quant_exact(x3, s)));
}

// Quantises 4 values; returns the 4 int8 results packed little-endian.
__device__ __forceinline__ uint32_t quant4(float x0, float x1, float x2, float x3, float s,
                                           float inv_s) {
  const float x[4] = {x0, x1, x2, x3};
  uint32_t t[4];
  bool ok = inv_s != 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float tf = __fmaf_rn(x[j], inv_s, kRoundMagic);
    const float d = __fmaf_rn(x[j], inv_s, -__fsub_rn(tf, kRoundMagic));
    ok = ok && (fabsf(d) <= kTieGuard);
    t[j] = __float_as_uint(tf);
  }
  if (__builtin_expect(!ok, 0)) return quant4_exact(x0, x1, x2, x3, s);
  return pack4_low_bytes(t[0], t[1], t[2], t[3]);
}

// Quantises 8 values; returns the 8 int8 results packed little-endian.
__device__ __forceinline__ uint2 quant8(const float (&x)[8], float s, float inv_s) {
  return make_uint2(quant4(x[0], x[1], x[2], x[3], s, inv_s),
                    quant4(x[4], x[5], x[6], x[7], s, inv_s));
}

// bf16 -> fp32 of the two halves of a packed pair (exact: bf16 is the top half
// of an fp32).
__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// Quantises the 8 bf16 of a 16-byte vector.
__device__ __forceinline__ uint2 quant8_bf16(const uint4& v, float s, float inv_s) {
  const float x[8] = {bf16_lo(v.x), bf16_hi(v.x), bf16_lo(v.y), bf16_hi(v.y),
                      bf16_lo(v.z), bf16_hi(v.z), bf16_lo(v.w), bf16_hi(v.w)};
  return quant8(x, s, inv_s);
}

}  // namespace lema
