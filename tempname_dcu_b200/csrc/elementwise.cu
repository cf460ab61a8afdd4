// Small memory-bound kernels of the tensor-parallel layer:
//   * out = x + bias[col] + residual            (after a reduce-scatter)
//   * deterministic column sums (bias gradients): per-CTA partial sums over
//     a fixed row range, then an ordered reduction of the partials added to
//     the fp32 accumulator (colred.cuh for 16-byte aligned rows, a 4-byte
//     variant otherwise).
//
// Reference parity: python/flux_dcu/model.py:257-263 (row-parallel output +
// replicated bias + residual) and the bias gradients autograd produces for
// ColumnLinear (:125) and the replicated biases.
#include "colred.cuh"
#include "common.cuh"

namespace tdb {
namespace ew {

__global__ void bias_residual_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ bias,
                                     const uint16_t* __restrict__ res, uint16_t* __restrict__ out, int64_t rows,
                                     int cols) {
  const int64_t n8 = rows * cols / 8;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n8; i += int64_t(gridDim.x) * blockDim.x) {
    const int col = int((i * 8) % cols);
    const uint4 a = reinterpret_cast<const uint4*>(x)[i];
    const uint4 r = res ? reinterpret_cast<const uint4*>(res)[i] : make_uint4(0, 0, 0, 0);
    const uint4 b = bias ? *reinterpret_cast<const uint4*>(bias + col) : make_uint4(0, 0, 0, 0);
    const uint32_t aa[4] = {a.x, a.y, a.z, a.w}, rr[4] = {r.x, r.y, r.z, r.w}, bb[4] = {b.x, b.y, b.z, b.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float lo = bf16_bits_to_float(aa[j] & 0xffff) + bf16_bits_to_float(bb[j] & 0xffff) +
                       bf16_bits_to_float(rr[j] & 0xffff);
      const float hi = bf16_bits_to_float(aa[j] >> 16) + bf16_bits_to_float(bb[j] >> 16) +
                       bf16_bits_to_float(rr[j] >> 16);
      o[j] = pack_bf16x2(lo, hi);
    }
    reinterpret_cast<uint4*>(out)[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

constexpr int kColRows = 64;  // rows per partial

// partial[p, c] = sum_{r in [p*64, p*64+64)} x[r, c]   (bf16 input)
__global__ void colsum_partial_kernel(const uint16_t* __restrict__ x, int64_t ld, int rows, int cols,
                                      float* __restrict__ partial) {
  const int c2 = (blockIdx.x * blockDim.x + threadIdx.x) * 2;
  const int p = blockIdx.y;
  if (c2 >= cols) return;
  float s0 = 0.f, s1 = 0.f;
  const int r1 = min(rows, (p + 1) * kColRows);
  for (int r = p * kColRows; r < r1; ++r) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(x + int64_t(r) * ld + c2);
    s0 += bf16_bits_to_float(w & 0xffff);
    s1 += bf16_bits_to_float(w >> 16);
  }
  partial[int64_t(p) * cols + c2] = s0;
  if (c2 + 1 < cols) partial[int64_t(p) * cols + c2 + 1] = s1;
}

__global__ void colsum_finish_kernel(const float* __restrict__ partial, int nparts, int cols, float* __restrict__ out,
                                     int accumulate) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  float s = 0.f;
  for (int p = 0; p < nparts; ++p) s += partial[int64_t(p) * cols + c];
  out[c] = accumulate ? out[c] + s : s;
}

}  // namespace ew
}  // namespace tdb

using namespace tdb::ew;

TDB_API int tdb_bias_residual(const void* x, const void* bias, const void* res, void* out, int64_t rows, int cols,
                              void* stream) {
  if (cols % 8) return tdb_host::fail(int(cudaErrorInvalidValue), "bias_residual: cols must be a multiple of 8");
  const int64_t n8 = rows * cols / 8;
  const int grid = int(n8 / 256 + 1 < 4096 ? n8 / 256 + 1 : 4096);
  bias_residual_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(bias), static_cast<const uint16_t*>(res),
      static_cast<uint16_t*>(out), rows, cols);
  tdb_host::launched(1);
  return int(cudaGetLastError());
}

// Scratch for tdb_colsum in floats: ceil(rows / 16) * cols covers either path
// below (the 16-byte path uses parts of at least 16 rows).
TDB_API int tdb_colsum_scratch_floats(int rows, int cols) { return ((rows + 15) / 16) * cols; }

TDB_API int tdb_colsum(const void* x, int64_t ld, int rows, int cols, float* partial, float* out, int accumulate,
                       void* stream) {
  if (cols % 2 || ld % 2 || rows <= 0) return tdb_host::fail(int(cudaErrorInvalidValue), "colsum: bad shape");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool wide = cols % 8 == 0 && ld % 8 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(partial) % 16 == 0;
  if (wide) {
    // 16-byte loads, a few waves of CTAs (colred.cuh)
    const int rpp = tdb::colred::rows_per_part(rows, cols, tdb_host::sm_count());
    const int nparts = (rows + rpp - 1) / rpp;
    if (int64_t(nparts) * cols <= int64_t(tdb_colsum_scratch_floats(rows, cols))) {
      dim3 g1((cols + tdb::colred::kColsPerCta - 1) / tdb::colred::kColsPerCta, nparts);
      tdb::colred::colred_partial<false><<<g1, tdb::colred::kThreads, 0, s>>>(
          static_cast<const uint16_t*>(x), ld, nullptr, 0, nullptr, nullptr, rows, cols, rpp, partial);
      tdb_host::launched(1);
      // one quantity (grid y = 1): only out0 is written
      tdb::colred::colred_finish<<<dim3((cols + 63) / 64, 1), 256, 0, s>>>(partial, nparts, cols, out, nullptr,
                                                                          accumulate);
      tdb_host::launched(1);
      return int(cudaGetLastError());
    }
  }
  const int nparts = (rows + kColRows - 1) / kColRows;
  dim3 grid((cols / 2 + 255) / 256, nparts);
  colsum_partial_kernel<<<grid, 256, 0, s>>>(static_cast<const uint16_t*>(x), ld, rows, cols, partial);
  tdb_host::launched(1);
  colsum_finish_kernel<<<(cols + 255) / 256, 256, 0, s>>>(partial, nparts, cols, out, accumulate);
  tdb_host::launched(1);
  return int(cudaGetLastError());
}
