// TACO H128 / E4M3FN codec building blocks (device functions).
//
// Wire format (identical to the reference, python/flux_dcu/codec.py:112-118 and
// src/taco/codec.hip:78-135): for E elements (E % 128 == 0, G = E/128 groups)
//   [E payload bytes, E4M3FN][G fp32 quant scales][G fp32 adaptive scales]
// so 136 bytes per 128-element group.  Per group:
//   a = clamp(448 * rsqrt(max(mean(x^2) + 1e-6, 1e-12)), 1e-3, 1e3)
//   u = H128(a * x) / sqrt(128)            (Sylvester-ordered Walsh-Hadamard)
//   q = clamp(max(max|u|, 1e-12) / 448, 1e-12, 1e6)
//   payload = e4m3_rne_satfinite(clamp(u_finite / q, -448, 448))
// and decode is x' = bf16(H128(e4m3(p) * q) / sqrt(128) / max(a, 1e-12)).
//
// Layout used here: one warp owns one group, lane L holds coefficients
// 4L..4L+3.  Butterfly strides 1 and 2 stay inside a thread; strides 4..64
// are lane-xor shuffles with masks 1..16.
#pragma once
#include <cuda_fp16.h>
#include <string.h>

#include "common.cuh"

namespace tdb {
namespace taco {

constexpr int kGroup = 128;
constexpr int kGroupBytes = 136;
constexpr float kInvSqrt128 = 0.08838834764831844055f;

// Two fp32 -> packed E4M3FN pair (round to nearest even, saturate to +-448).
// Byte 0 holds `lo`, byte 1 holds `hi`.
__device__ __forceinline__ uint16_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

__host__ __device__ __forceinline__ float bits_as_float(uint32_t u) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  float f;
  memcpy(&f, &u, 4);
  return f;
#endif
}

// E4M3FN code -> fp32 (exact).  0x7f / 0xff are NaN in E4M3FN.
__host__ __device__ __forceinline__ float e4m3_to_float(uint32_t code) {
  const uint32_t mag = code & 0x7fu;
  float v;
  if (mag == 0x7fu) {
    v = bits_as_float(0x7fc00000u);
  } else if (mag < 8u) {
    v = float(mag) * 0.001953125f;  // subnormal: mag * 2^-9
  } else {
    // normal: exponent field e = mag>>3 (bias 7), mantissa m = mag&7
    // value = (1 + m/8) * 2^(e-7) -> build the fp32 bit pattern directly
    const uint32_t e = (mag >> 3) + 120u;  // 127 - 7
    v = bits_as_float((e << 23) | ((mag & 7u) << 20));
  }
  return (code & 0x80u) ? -v : v;
}

// Four E4M3FN codes packed in a word (code j in byte j) -> fp32, with the
// hardware conversion (two codes per instruction into f16, exact: every E4M3
// value, NaN included, is representable in f16).  Same values as
// e4m3_to_float, which stays the host-testable definition.
__device__ __forceinline__ void e4m3x4_to_float(uint32_t word, float (&out)[4]) {
  uint32_t lo, hi;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(lo) : "h"(uint16_t(word & 0xffffu)));
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(hi) : "h"(uint16_t(word >> 16)));
  const __half2 a = *reinterpret_cast<const __half2*>(&lo), b = *reinterpret_cast<const __half2*>(&hi);
  out[0] = __low2float(a);
  out[1] = __high2float(a);
  out[2] = __low2float(b);
  out[3] = __high2float(b);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// In-place unnormalised H128 over a warp; lane holds x[0..3] = coefficients
// 4*lane + 0..3.
__device__ __forceinline__ void fwht128_warp(float (&x)[4], int lane) {
  // stride 1
  {
    float a = x[0], b = x[1];
    x[0] = a + b; x[1] = a - b;
    a = x[2]; b = x[3];
    x[2] = a + b; x[3] = a - b;
  }
  // stride 2
  {
    float a = x[0], b = x[2];
    x[0] = a + b; x[2] = a - b;
    a = x[1]; b = x[3];
    x[1] = a + b; x[3] = a - b;
  }
  // strides 4..64 -> lane masks 1..16
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const bool upper = (lane & m) != 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float other = __shfl_xor_sync(0xffffffffu, x[j], m);
      x[j] = upper ? (other - x[j]) : (x[j] + other);
    }
  }
}

struct GroupScales {
  float quant;
  float adaptive;
};

// Encode one group held by a warp.  Returns the packed 4 payload bytes of
// this lane (coefficient 4*lane in byte 0) and the two scales (same on all
// lanes).
__device__ __forceinline__ uint32_t encode_group_warp(const float (&in)[4], int lane, GroupScales& s) {
  float x[4];
  float sq = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) sq += in[j] * in[j];
  sq = warp_sum(sq);
  const float variance = fmaxf(sq * (1.0f / 128.0f) + 1e-6f, 1e-12f);
  const float a = fminf(fmaxf(448.0f * rsqrtf(variance), 1e-3f), 1e3f);
#pragma unroll
  for (int j = 0; j < 4; ++j) x[j] = in[j] * a;
  fwht128_warp(x, lane);
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    x[j] *= kInvSqrt128;
    amax = fmaxf(amax, fabsf(x[j]));
  }
  amax = warp_max(amax);
  const float q = fminf(fmaxf(fmaxf(amax, 1e-12f) / 448.0f, 1e-12f), 1e6f);
  float y[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float f = isfinite(x[j]) ? x[j] : 0.0f;
    y[j] = fminf(fmaxf(f / q, -448.0f), 448.0f);
  }
  s.quant = q;
  s.adaptive = a;
  return uint32_t(e4m3x2(y[0], y[1])) | (uint32_t(e4m3x2(y[2], y[3])) << 16);
}

// Decode one group held by a warp: payload word (4 codes, coefficient 4*lane
// in byte 0) -> 4 fp32 values (already divided by the adaptive scale).
__device__ __forceinline__ void decode_group_warp(uint32_t payload, float quant, float adaptive, int lane,
                                                  float (&out)[4]) {
  e4m3x4_to_float(payload, out);
#pragma unroll
  for (int j = 0; j < 4; ++j) out[j] *= quant;
  fwht128_warp(out, lane);
  const float den = fmaxf(adaptive, 1e-12f);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float v = out[j] * kInvSqrt128;
    out[j] = (isfinite(v) ? v : 0.0f) / den;
  }
}

}  // namespace taco
}  // namespace tdb
