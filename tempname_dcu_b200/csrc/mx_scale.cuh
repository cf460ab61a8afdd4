// Scale rule of the block-scaled FP8 (MXFP8) quantizer, shared by the device
// quantizer (gemm_mx.cu) and host builds of the same function (tests compile
// it with the host compiler and check it exhaustively over bf16 inputs).
//
// For a 32-value block with absolute maximum `amax`, the exponent is the
// smallest e with amax * 2^-e <= 448 (the largest finite e4m3), so no value
// saturates; it is clamped to the ue8m0 range [-127, 127].  Zero and
// subnormal maxima use the smallest scale.
#pragma once
#include <cstdint>
#include <cstring>

namespace tdb {
namespace mx_scale {

__host__ __device__ __forceinline__ int block_exponent(float amax) {
  uint32_t bits;
#ifdef __CUDA_ARCH__
  bits = __float_as_uint(amax);
#else
  std::memcpy(&bits, &amax, 4);
#endif
  const int field = int((bits >> 23) & 0xFF);
  if (field == 0) return -127;
  // amax = (1 + f) 2^E;  448 = 1.75 * 2^8
  const int e = field - 127 - 8 + ((bits & 0x7FFFFF) > 0x600000 ? 1 : 0);
  return e < -127 ? -127 : (e > 127 ? 127 : e);
}

}  // namespace mx_scale
}  // namespace tdb
