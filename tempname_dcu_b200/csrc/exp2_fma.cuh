// 2^x without the special-function unit, for a share of the softmax
// exponentials (which would otherwise all queue on the MUFU/XU pipe, shared
// with the float <-> bf16 conversions):
//   n = round(x) by the shifter-constant trick (x + 1.5 * 2^23 leaves n in the
//   low mantissa bits; an FADD, not an F2I conversion), f = x - n in
//   [-0.5, 0.5], 2^x = 2^n * p(f),
// where p is the cubic interpolating 2^f at the four Chebyshev points of the
// first kind on [-0.5, 0.5] (Chebyshev interpolation; monomial coefficients
// from the 4 x 4 Vandermonde system at those nodes; max relative error
// 1.0e-4 on the interval, below the bf16 rounding of the probabilities it
// feeds).  2^n is added to p's exponent field with one integer multiply-add
// of t's bits (t's bits times 2^23 keep exactly n << 23 modulo 2^32).
// Arguments are <= 0 in the softmax; they are clamped at -125, so anything
// smaller returns 2^-125 (negligible next to the row maximum's 1).
// Host and device: tests/test_exp2_fma_host.py checks it against exp2.
#pragma once
#include <math.h>
#include <stdint.h>
#include <string.h>

namespace tdb {

__host__ __device__ __forceinline__ float exp2_fma(float x) {
  constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
  x = fmaxf(x, -125.0f);
  const float t = x + kShift;
  const float f = x - (t - kShift);
  const float p = fmaf(fmaf(fmaf(0.05583828f, f, 0.24263948f), f, 0.69313675f), f, 0.99992454f);
#ifdef __CUDA_ARCH__
  return __uint_as_float(__float_as_uint(t) * (1u << 23) + __float_as_uint(p));
#else
  uint32_t tb, pb;
  memcpy(&tb, &t, 4);
  memcpy(&pb, &p, 4);
  const uint32_t yb = tb * (1u << 23) + pb;
  float y;
  memcpy(&y, &yb, 4);
  return y;
#endif
}

}  // namespace tdb
