// openTPU fp32 arithmetic on the GPU: round-to-nearest-even, flush-to-zero on operands and on
// results, canonical NaN 0x7FC00000 (reference docs/isa.md "Arithmetic (fp32)",
// opentpu/fp32.py:45-101).
//
// This translation unit is compiled WITHOUT -ftz (IEEE subnormals on), so __fmul_rn rounds a
// tiny product onto the subnormal grid first and otq_flush then decides: a product that
// rounds up to 2^-126 is a normal number and is kept (tests/test_fp.py:214). The *_rn
// intrinsics are never contracted into an FMA.
#pragma once
#include <cstdint>

namespace otq {

__device__ __forceinline__ float otq_flush(float x) {
  uint32_t b = __float_as_uint(x);
  return ((b & 0x7F800000u) == 0u) ? __uint_as_float(b & 0x80000000u) : x;
}

__device__ __forceinline__ float otq_canon(float x) {
  return (x != x) ? __uint_as_float(0x7FC00000u) : x;
}

__device__ __forceinline__ float fmul(float a, float b) {
  return otq_canon(otq_flush(__fmul_rn(otq_flush(a), otq_flush(b))));
}

__device__ __forceinline__ float fadd(float a, float b) {
  return otq_canon(otq_flush(__fadd_rn(otq_flush(a), otq_flush(b))));
}

__device__ __forceinline__ float fsub(float a, float b) {
  return otq_canon(otq_flush(__fsub_rn(otq_flush(a), otq_flush(b))));
}

// openTPU's reciprocal (docs/isa.md "recip", opentpu/fp32.py:242-261): on the significand
// a in [1, 2) a magic seed, two Newton steps y*(2 - a*y), the correction step
// y*(1 - a*y) + y, then 127 - field(x) added to y's exponent field and x's sign or-ed in.
// Zero -> +0; |x| >= 2^126 (inf and NaN included) -> a zero with x's sign.
// On the significand every operand and result of the steps is a normal number or zero (the
// seed lies in (0.47, 0.96), a*y and the Newton factors near 1, the correction term a multiple
// of 2^-24 times y), so the flushes and the NaN canonicalisation of fmul / fsub /
// fadd are no-ops there and plain round-to-nearest operations give the same bits.
__device__ __forceinline__ float recip(float x) {
  const uint32_t xb = __float_as_uint(otq_flush(x));
  const uint32_t mag = xb & 0x7FFFFFFFu;
  const uint32_t sign = xb & 0x80000000u;
  if (mag == 0u) return 0.0f;
  if (mag >= 0x7E800000u) return __uint_as_float(sign);
  const float a = __uint_as_float(0x3F800000u | (mag & 0x007FFFFFu));
  float y = __uint_as_float(0x7EF311C3u - __float_as_uint(a));
  y = __fmul_rn(y, __fsub_rn(2.0f, __fmul_rn(a, y)));
  y = __fmul_rn(y, __fsub_rn(2.0f, __fmul_rn(a, y)));
  y = __fadd_rn(__fmul_rn(y, __fsub_rn(1.0f, __fmul_rn(a, y))), y);
  const int k = 127 - static_cast<int>(mag >> 23);
  const uint32_t yb = static_cast<uint32_t>(static_cast<int>(__float_as_uint(y)) + k * (1 << 23));
  return __uint_as_float(yb | sign);
}

// q8: round half to even, clip to [-127, 127], NaN -> 0 (opentpu/fp32.py:167-172).
__device__ __forceinline__ int q8(float p) {
  p = otq_flush(p);
  if (p != p) return 0;
  float r = rintf(p);
  r = fminf(fmaxf(r, -127.0f), 127.0f);
  return static_cast<int>(r);
}

// The largest d <= 31 with a * 2^d <= amax from the two magnitude bit patterns
// (opentpu/fp32.py:313-318); 0 where a == 0.
__device__ __forceinline__ int group_offset(uint32_t a, uint32_t amax) {
  if (a == 0u) return 0;
  int d = static_cast<int>(amax >> 23) - static_cast<int>(a >> 23) -
          ((a & 0x7FFFFFu) > (amax & 0x7FFFFFu) ? 1 : 0);
  return d < 0 ? 0 : (d > 31 ? 31 : d);
}

// f32(1/127), the quantizer's scale factor (opentpu/fp32.py:28 INV127).
constexpr uint32_t kInv127Bits = 0x3C010204u;

// 2^d as fp32 for 0 <= d <= 31.
__device__ __forceinline__ float pow2i(int d) { return __uint_as_float((127u + d) << 23); }

// The MM epilogue (docs/isa.md "MM"; opentpu/isasim.py:899-900):
// y = (i2f(acc) * Sw) * (Sa * 2^-W), three flushed RNE products, i2f round-to-nearest-even.
__device__ __forceinline__ float mm_epilogue(long long acc, float Sw, float Sa, int W) {
  const float inv_w = __uint_as_float(static_cast<uint32_t>(127 - W) << 23);
  return fmul(fmul(__ll2float_rn(acc), Sw), fmul(Sa, inv_w));
}

}  // namespace otq
