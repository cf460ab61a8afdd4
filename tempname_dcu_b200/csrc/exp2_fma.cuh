// 2^x on the FMA pipe, for a share of the softmax exponentials (which would
// otherwise all queue on the special-function unit):
//   x = n + f, n = floor(x), f in [0, 1);  2^x = 2^n * p(f),
// where p is the cubic that interpolates 2^f at the four Chebyshev points of
// the first kind on [0, 1] (Chebyshev interpolation; the monomial
// coefficients below were computed offline by solving the 4 x 4 Vandermonde
// system at those nodes; max relative error 1.0e-4 on [0, 1], well below the
// bf16 rounding of the probabilities it feeds), and 2^n is added to p's
// exponent bits.  Arguments are <= 0 in the softmax; below -125 the result
// is 0 (such contributions vanish in bf16, as with a flush-to-zero ex2).
// Host and device: tests/test_exp2_fma_host.py checks it against exp2.
#pragma once
#include <math.h>
#include <stdint.h>
#include <string.h>

namespace tdb {

__host__ __device__ __forceinline__ float exp2_fma(float x) {
  const float n = floorf(x);
  const float f = x - n;
  const float p = fmaf(fmaf(fmaf(0.07896726f, f, 0.22469315f), f, 0.69632477f), f, 0.99990028f);
#ifdef __CUDA_ARCH__
  const float y = __int_as_float(__float_as_int(p) + (int(n) << 23));
#else
  int32_t bits;
  memcpy(&bits, &p, 4);
  bits += int32_t(n) * (1 << 23);
  float y;
  memcpy(&y, &bits, 4);
#endif
  return x < -125.f ? 0.f : y;
}

}  // namespace tdb
