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
// The fast form takes t = rint(x * RN(1/s)) while |d| = |x * RN(1/s) - t| <=
// kTieGuard. For |x / s| <= 127.5 the exact product x * RN(1/s) is within
// 127.5 * 2^-24 (7.6e-6) of x / s, the contract's fp32 quotient RN(x / s) within
// 2^-18 (3.8e-6) of x / s, and d carries one more rounding (2^-25): the two
// round to the same integer whenever |d| <= 0.5 - 1.2e-5. The guard keeps a
// margin of 2e-5.
constexpr float kTieGuard = 0.49998f;

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

// ---- packed fp32 pairs (sm_100: one instruction computes two fp32 lanes) ----

__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

// a * b + c per lane, each rounded once (round to nearest even).
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ uint64_t f2_splat(float v) { return f2_pack(v, v); }

// The two bf16 of a 32-bit word (low half first) as an fp32 pair.
__device__ __forceinline__ uint64_t f2_from_bf16x2(uint32_t w) {
  return f2_pack(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

// An fp32 pair rounded (to nearest even) to two bf16 in one word, low half first.
__device__ __forceinline__ uint32_t bf16x2_from_f2(uint64_t v) {
  float lo, hi;
  f2_unpack(v, lo, hi);
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// max(m, |a|), NaN if either is NaN.
__device__ __forceinline__ float max_abs_nan(float m, float a) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(m), "f"(fabsf(a)));
  return r;
}

// The fast form for 4 values held as two fp32 pairs, two elements per
// instruction: t = RN(x * inv_s + 1.5 * 2^23) (its low byte is the candidate),
// d = RN(x * inv_s - (t - 1.5 * 2^23)) (the distance to it, exact up to one
// fp32 rounding). Folds max |d| into dmax (NaN-propagating); the caller takes
// the candidates only while dmax <= kTieGuard and inv_s != 0.
__device__ __forceinline__ uint32_t quant4_fast(uint64_t x01, uint64_t x23, uint64_t inv2,
                                                float& dmax) {
  const uint64_t mag2 = f2_splat(kRoundMagic);
  const uint64_t neg1 = f2_splat(-1.f);
  const uint64_t t01 = f2_fma(x01, inv2, mag2);
  const uint64_t t23 = f2_fma(x23, inv2, mag2);
  const uint64_t d01 = f2_fma(x01, inv2, f2_fma(t01, neg1, mag2));
  const uint64_t d23 = f2_fma(x23, inv2, f2_fma(t23, neg1, mag2));
  float d0, d1, d2, d3, t0, t1, t2, t3;
  f2_unpack(d01, d0, d1);
  f2_unpack(d23, d2, d3);
  dmax = max_abs_nan(max_abs_nan(dmax, d0), d1);
  dmax = max_abs_nan(max_abs_nan(dmax, d2), d3);
  f2_unpack(t01, t0, t1);
  f2_unpack(t23, t2, t3);
  return pack4_low_bytes(__float_as_uint(t0), __float_as_uint(t1), __float_as_uint(t2),
                         __float_as_uint(t3));
}

// Quantises 4 values held as two fp32 pairs: the fast form, or the exact
// division for all 4 when one of them is within the guard of a tie (bf16 rows
// sit on a coarse grid, so exact ties are common: about 1 element in 3000 of
// Gaussian rows) or when fast_ok (inv_s != 0) is false. Checked per 4 values so
// that a tie costs its warp 4 divisions.
__device__ __forceinline__ uint32_t quant4_pairs(uint64_t x01, uint64_t x23, uint64_t inv2,
                                                 float s, bool fast_ok) {
  float dmax = 0.f;
  const uint32_t r = quant4_fast(x01, x23, inv2, dmax);
  if (__builtin_expect(!(dmax <= kTieGuard) || !fast_ok, 0)) {
    float x0, x1, x2, x3;
    f2_unpack(x01, x0, x1);
    f2_unpack(x23, x2, x3);
    return quant4_exact(x0, x1, x2, x3, s);
  }
  return r;
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
  const uint64_t inv2 = f2_splat(inv_s);
  const bool fast_ok = inv_s != 0.f;
  return make_uint2(quant4_pairs(f2_from_bf16x2(v.x), f2_from_bf16x2(v.y), inv2, s, fast_ok),
                    quant4_pairs(f2_from_bf16x2(v.z), f2_from_bf16x2(v.w), inv2, s, fast_ok));
}

}  // namespace lema
