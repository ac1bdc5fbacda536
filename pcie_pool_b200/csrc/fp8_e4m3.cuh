// bf16 / fp32 -> fp8 e4m3 codes of x / scale, as if the quotient were first
// rounded to fp32 (IEEE round-to-nearest-even) and then converted with
// cvt.rn.satfinite.e4m3x2.f32.
//
// A correctly rounded fp32 division per element is an instruction sequence
// with a data-dependent branch; at 16384 elements per 128x128 block it bound
// the quantizer to a few percent of HBM bandwidth.  The e4m3 code depends only
// on which side of an e4m3 rounding boundary the quotient falls, so the
// quotient is estimated as q = x * r with r = 1/scale (one correctly rounded
// reciprocal per block) and the division is done only when the estimate is
// too close to a boundary to decide -- Ziv's strategy ("Fast evaluation of
// elementary mathematical functions with correctly rounded last bit", ACM
// TOMS 17(3), 1991): compute cheaply with an error bound, fall back to the
// exact operation when the bound does not settle the rounding.
//
// Error bound: r = (1/s)(1+d1), q = x r (1+d2), |d1|, |d2| <= 2^-24, and the
// correctly rounded quotient Q = (x/s)(1+d3), |d3| <= 2^-24, so |q - Q| <=
// 3 * 2^-24 |x/s| (+ 2^-149 absolute when q is subnormal) -- at most 3 ulps
// in one binade, 6 when q and Q straddle a power of two.  Positive floats
// are ordered like their bit patterns, so Q lies between the floats 8 steps
// below and above |q|; the conversion is monotone, so when both ends convert
// to the same code, Q does too.  The signs are applied to the magnitude codes
// (the conversion is odd: code(-a) = code(a) | 0x80, zero included).  A
// reciprocal that overflows (a subnormal scale) sends the block to the exact
// path.  Checked bit-exact against the division-based CPU quantizer by the
// tests (random blocks and blocks of exact midpoints).
#pragma once

#include <cuda_fp8.h>

#include <cstdint>

namespace ppb {

__device__ __forceinline__ uint32_t e4m3x2_code(float a, float b) {
  return static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3));
}

// The rare exact path, kept out of line so the unrolled hot loops that call
// e4m3x2_quotient stay small (inlined divisions filled the instruction cache).
static __device__ __noinline__ uint32_t e4m3x2_settle(uint32_t mag, uint32_t diff, float x0, float x1, float s) {
  if (diff & 0x00ffu) mag = (mag & 0xff00u) | (e4m3x2_code(__fdiv_rn(fabsf(x0), s), 0.f) & 0x00ffu);
  if (diff & 0xff00u) mag = (mag & 0x00ffu) | (e4m3x2_code(0.f, __fdiv_rn(fabsf(x1), s)) & 0xff00u);
  return mag;
}

static __device__ __noinline__ uint32_t e4m3x2_divide(float x0, float x1, float s) {
  return e4m3x2_code(__fdiv_rn(x0, s), __fdiv_rn(x1, s));
}

// Two e4m3 codes (x0 in the low byte) of x0 / s and x1 / s; r = __frcp_rn(s).
__device__ __forceinline__ uint32_t e4m3x2_quotient(float x0, float x1, float s, float r, bool exact_only) {
  if (exact_only) return e4m3x2_divide(x0, x1, s);
  const float q0 = __fmul_rn(x0, r);
  const float q1 = __fmul_rn(x1, r);
  const uint32_t b0 = __float_as_uint(q0), b1 = __float_as_uint(q1);
  const uint32_t a0 = b0 & 0x7fffffffu, a1 = b1 & 0x7fffffffu;
  const uint32_t lo = e4m3x2_code(__uint_as_float(a0 > 8u ? a0 - 8u : 0u), __uint_as_float(a1 > 8u ? a1 - 8u : 0u));
  const uint32_t hi = e4m3x2_code(__uint_as_float(a0 + 8u), __uint_as_float(a1 + 8u));
  const uint32_t diff = lo ^ hi;
  // rare: an estimate within 8 ulps of a rounding boundary
  const uint32_t mag = diff ? e4m3x2_settle(lo, diff, x0, x1, s) : lo;
  return mag | ((b0 >> 24) & 0x80u) | ((b1 >> 16) & 0x8000u);
}

}  // namespace ppb
