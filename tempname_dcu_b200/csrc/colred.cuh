// Deterministic column reductions over the rows of bf16 matrices, shared by
// the bias gradients (sum_r dy[r, c]) and the LayerNorm parameter gradients
// (sum_r dy[r, c] * xhat[r, c] and sum_r dy[r, c]).
//
// Stage 1 (colred_partial): CTA = 256 threads x 8 columns (one 16-byte load
// per row and thread), over a fixed block of rows; writes fp32 partials
// [quantity][part][cols].  Stage 2 (colred_finish): CTA = 8 warps over 64
// columns; warp w adds parts w, w+8, ... and the eight warp sums are combined
// in warp order.  Every sum has a fixed order, so results are bitwise
// reproducible; no floating-point atomics.
#pragma once
#include "common.cuh"

namespace tdb {
namespace colred {

constexpr int kThreads = 256;
constexpr int kColsPerCta = kThreads * 8;

__device__ __forceinline__ void unpack8(const uint4 w, float (&v)[8]) {
  const uint32_t a[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    v[2 * j] = bf16_bits_to_float(a[j] & 0xffff);
    v[2 * j + 1] = bf16_bits_to_float(a[j] >> 16);
  }
}

// LN = false: partial[0][p][c] = sum_{r in part p} dy[r, c]
// LN = true:  partial[0][p][c] = sum dy * (x - mean_r) * rstd_r, partial[1][p][c] = sum dy
template <bool LN>
__global__ void __launch_bounds__(kThreads) colred_partial(const uint16_t* __restrict__ dy, int64_t ld_dy,
                                                           const uint16_t* __restrict__ x, int64_t ld_x,
                                                           const float* __restrict__ mean,
                                                           const float* __restrict__ rstd, int rows, int cols,
                                                           int rows_per_part, float* __restrict__ partial) {
  const int c8 = (blockIdx.x * kThreads + threadIdx.x) * 8;
  if (c8 >= cols) return;
  const int p = blockIdx.y, nparts = gridDim.y;
  const int r0 = p * rows_per_part, r1 = min(rows, r0 + rows_per_part);
  float a[8], b[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) a[j] = b[j] = 0.f;
#pragma unroll 4
  for (int r = r0; r < r1; ++r) {
    float d[8];
    unpack8(*reinterpret_cast<const uint4*>(dy + int64_t(r) * ld_dy + c8), d);
    if (LN) {
      float xv[8];
      unpack8(*reinterpret_cast<const uint4*>(x + int64_t(r) * ld_x + c8), xv);
      const float mu = mean[r], rs = rstd[r];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        a[j] += d[j] * ((xv[j] - mu) * rs);
        b[j] += d[j];
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] += d[j];
    }
  }
  float4* pa = reinterpret_cast<float4*>(partial + int64_t(p) * cols + c8);
  pa[0] = make_float4(a[0], a[1], a[2], a[3]);
  pa[1] = make_float4(a[4], a[5], a[6], a[7]);
  if (LN) {
    float4* pb = reinterpret_cast<float4*>(partial + (int64_t(nparts) + p) * cols + c8);
    pb[0] = make_float4(b[0], b[1], b[2], b[3]);
    pb[1] = make_float4(b[4], b[5], b[6], b[7]);
  }
}

// out_q[c] (+)= sum_p partial[q][p][c] for q = blockIdx.y (out0 / out1).
static __global__ void __launch_bounds__(256) colred_finish(const float* __restrict__ partial, int nparts, int cols,
                                                     float* __restrict__ out0, float* __restrict__ out1,
                                                     int accumulate) {
  __shared__ float2 acc[8][32];
  const int q = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x * 64 + lane * 2;
  const float* src = partial + int64_t(q) * nparts * cols;
  float2 s = make_float2(0.f, 0.f);
  if (c < cols) {
    int p = warp;
    for (; p + 24 < nparts; p += 32) {  // four loads in flight, added in part order
      float2 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = *reinterpret_cast<const float2*>(src + int64_t(p + 8 * u) * cols + c);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        s.x += v[u].x;
        s.y += v[u].y;
      }
    }
    for (; p < nparts; p += 8) {
      const float2 v = *reinterpret_cast<const float2*>(src + int64_t(p) * cols + c);
      s.x += v.x;
      s.y += v.y;
    }
  }
  acc[warp][lane] = s;
  __syncthreads();
  if (warp == 0 && c < cols) {
    float2 t = acc[0][lane];
#pragma unroll
    for (int w = 1; w < 8; ++w) {
      t.x += acc[w][lane].x;
      t.y += acc[w][lane].y;
    }
    float* out = q == 0 ? out0 : out1;
    if (accumulate) {
      out[c] += t.x;
      out[c + 1] += t.y;
    } else {
      out[c] = t.x;
      out[c + 1] = t.y;
    }
  }
}

// Rows per partial so that stage 1 has a few waves of CTAs.
inline int rows_per_part(int rows, int cols, int sms) {
  const int col_ctas = (cols + kColsPerCta - 1) / kColsPerCta;
  int rpp = 16;
  while (rpp < rows && int64_t(col_ctas) * ((rows + rpp - 1) / rpp) > 4 * int64_t(sms)) rpp *= 2;
  return rpp;
}

}  // namespace colred
}  // namespace tdb
