// Block-scaled FP8 ("MX") GEMM on tcgen05 kind::mxf8f6f4 and its quantizer.
//
// Reference parity: the reference's selective arm (python/flux_dcu/runtime.py:
// 196-197, the per-physical-block mask of the calibrated plan) quantizes the
// selected output blocks on the wire only.  The B200 build can also run the
// selected blocks' GEMM itself in block-scaled FP8: e4m3 values with one
// power-of-two ue8m0 scale per 32 consecutive K values (the OCP Microscaling
// "MXFP8" format), accumulated in fp32 in TMEM.  This file holds the
// quantizer (bf16 -> e4m3 + scale atoms) and a standalone GEMM entry point;
// the same mainloop path (gemm_mainloop<..., MX = true>) serves the fused
// GEMM -> reduce-scatter kernel.
//
// Scale choice: for a 32-value block with absolute maximum a, the exponent is
// the smallest e with a * 2^-e <= 448 (the largest finite e4m3), so no value
// saturates; the stored byte is e + 127.  An all-zero block stores byte 0.
#include "gemm.cuh"
#include "gemm_epi.cuh"
#include "mx_scale.cuh"
#include "tensor_map.h"

namespace tdb {
namespace gemm {
namespace mx {

// 256-wide tiles (one TMEM accumulator, three stages) when N allows: at 128
// columns a K = 32 FP8 MMA reads as many shared-memory bytes per clock as the
// SM delivers, so only the wider tile lets FP8 outrun BF16.
template <int BN>
constexpr int kStagesFor = BN == 256 ? 3 : 5;

// Round-to-nearest-even, saturating fp32 pair -> e4m3 pair (low byte = lo).
__device__ __forceinline__ uint16_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("{\n\t.reg .b16 t;\n\tcvt.rn.satfinite.e4m3x2.f32 t, %2, %1;\n\tmov.b16 %0, t;\n\t}" : "=h"(r) : "f"(lo), "f"(hi));
  return r;
}

using mx_scale::block_exponent;  // the scale rule (mx_scale.cuh)

// One thread per (row, 32-value K block).  With `version` set the whole
// kernel is skipped while *version == *seen (the operand has not changed
// since it was last quantized); mark_kernel then records the version.
__global__ void __launch_bounds__(256) quantize_kernel(const uint16_t* __restrict__ x, int64_t ldx, int rows, int K,
                                                       uint8_t* __restrict__ q, uint8_t* __restrict__ sf,
                                                       const int* version, const int* seen) {
  if (version && __ldg(version) == *seen) return;
  const int64_t blocks_per_row = K / 32;
  const int64_t id = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (id >= int64_t(rows) * blocks_per_row) return;
  const int r = int(id / blocks_per_row);
  const int kb = int(id % blocks_per_row);
  const uint4* src = reinterpret_cast<const uint4*>(x + int64_t(r) * ldx + kb * 32);
  uint4 v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = src[i];
  const uint16_t* h = reinterpret_cast<const uint16_t*>(v);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(bf16_bits_to_float(h[i])));
  const int e = block_exponent(amax);
  const float inv = __uint_as_float(uint32_t(127 - e) << 23);  // 2^-e, a normal float for e in [-127, 126]
  uint4 out[2];
  uint16_t* o = reinterpret_cast<uint16_t*>(out);
#pragma unroll
  for (int i = 0; i < 16; ++i)
    o[i] = e4m3x2(bf16_bits_to_float(h[2 * i]) * inv, bf16_bits_to_float(h[2 * i + 1]) * inv);
  uint4* dst = reinterpret_cast<uint4*>(q + int64_t(r) * K + kb * 32);
  dst[0] = out[0];
  dst[1] = out[1];
  const int kc = kb / 4, j = kb % 4;
  const int64_t atom = int64_t(kc) * (rows / 128) + r / 128;
  sf[atom * 512 + (r % 32) * 16 + ((r % 128) / 32) * 4 + j] = uint8_t(e + 127);
}

__global__ void mark_kernel(const int* version, int* seen) { *seen = *version; }

template <int BN, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_mx_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int K,
                   TileOrder order, const __grid_constant__ EpiParams ep, const uint8_t* sfa, const uint8_t* sfb,
                   int a_blocks, int b_blocks, int* status) {
  typename EpiFor<MODE>::type epi{ep};
  MxOperands mxo{&tmA, &tmB, sfa, sfb, a_blocks, b_blocks, nullptr};
  gemm_mainloop<BN, false, false, typename EpiFor<MODE>::type, kStagesFor<BN>, true>(&tmA, &tmB, K, order, epi,
                                                                                    status, &mxo);
}

template <int BN, int MODE>
static int launch(const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K, const EpiParams& ep,
                  const uint8_t* sfa, const uint8_t* sfb, cudaStream_t stream) {
  using Cfg = Config<BN, kStagesFor<BN>, true>;
  constexpr int kSmem = Cfg::kSmemBytes + EpiFor<MODE>::type::kSmemBytes;
  static_assert(kSmem <= 227 * 1024, "shared memory budget");
  auto kern = gemm_mx_kernel<BN, MODE>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return tdb_host::fail(int(e), "cudaFuncSetAttribute(gemm_mx) failed");
    attr_set[dev & 63] = true;
  }
  TileOrder order;
  order.num_m = M / BM;
  order.num_n = N / BN;
  order.group_m = 16;
  order.table = nullptr;
  order.num_tiles = order.num_m * order.num_n;
  const int sms = tdb_host::grid_sms();
  const int grid = order.num_tiles < sms ? order.num_tiles : sms;
  kern<<<grid, kThreads, kSmem, stream>>>(ta, tb, K, order, ep, sfa, sfb, M / 128, N / 128, tdb_host::status_ptr());
  tdb_host::launched(1);
  return int(cudaGetLastError());
}

}  // namespace mx

// TMA map of an e4m3 operand [rows, K] (K-major, 128-byte swizzle), box
// {128 bytes, box_rows}.
int make_fp8_map(CUtensorMap* map, const void* ptr, int rows, int K, int box_rows) {
  return tdb_host::make_tmap_2d(map, ptr, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, uint64_t(K), uint64_t(rows), uint64_t(K),
                                128, uint32_t(box_rows), CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace gemm
}  // namespace tdb

using namespace tdb;
using namespace tdb::gemm;

// Bytes of the scale atoms of a [rows, K] operand.
TDB_API long long tdb_mx_scale_bytes(long long rows, long long K) { return rows / 128 * (K / 128) * 512; }

// x bf16 [rows, K] (row stride ldx) -> q e4m3 [rows, K] (dense) and scale
// atoms sf (tdb_mx_scale_bytes).  rows and K multiples of 128.
// With version / seen (device int32 scalars, or both null): quantize only
// when *version differs from *seen, then set *seen = *version -- e.g. a
// weight re-quantized once per optimizer step, also under CUDA graph replay.
TDB_API int tdb_mx_quantize_versioned(const void* x, long long ldx, int rows, int K, void* q, void* sf,
                                      const int* version, int* seen, void* stream) {
  if (!x || !q || !sf || rows <= 0 || K <= 0 || rows % 128 || K % 128 || ldx % 8 ||
      reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(q) % 16 || (!version != !seen))
    return tdb_host::fail(int(cudaErrorInvalidValue), "mx_quantize: rows and K must be multiples of 128, 16-byte rows");
  const int64_t n = int64_t(rows) * (K / 32);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  mx::quantize_kernel<<<unsigned((n + 255) / 256), 256, 0, s>>>(static_cast<const uint16_t*>(x), ldx, rows, K,
                                                                 static_cast<uint8_t*>(q), static_cast<uint8_t*>(sf),
                                                                 version, seen);
  tdb_host::launched(1);
  if (version) {
    mx::mark_kernel<<<1, 1, 0, s>>>(version, seen);
    tdb_host::launched(1);
  }
  return int(cudaGetLastError());
}

TDB_API int tdb_mx_quantize(const void* x, long long ldx, int rows, int K, void* q, void* sf, void* stream) {
  return tdb_mx_quantize_versioned(x, ldx, rows, K, q, sf, nullptr, nullptr, stream);
}

// C bf16 [M, N] (row stride ldc) = (A * 2^sfa) (B * 2^sfb)^T (+ bias[N] for
// mode 1): A e4m3 [M, K], B e4m3 [N, K], scales as written by
// tdb_mx_quantize.  M, N, K multiples of 128.
TDB_API int tdb_gemm_mx(const void* A, const void* sfa, const void* B, const void* sfb, void* C, long long ldc, int M,
                        int N, int K, int mode, const void* bias, void* stream) {
  if (!A || !B || !sfa || !sfb || !C || M <= 0 || N <= 0 || K <= 0 || M % 128 || N % 128 || K % 128 || ldc % 8 ||
      (mode != kStore && mode != kBias) || (mode == kBias && !bias))
    return tdb_host::fail(int(cudaErrorInvalidValue), "gemm_mx: M, N, K multiples of 128; mode 0 or 1 (with bias)");
  if ((reinterpret_cast<uintptr_t>(sfa) | reinterpret_cast<uintptr_t>(sfb)) % 16 ||
      (bias && reinterpret_cast<uintptr_t>(bias) % 16))
    return tdb_host::fail(int(cudaErrorInvalidValue), "gemm_mx: scales and bias must be 16-byte aligned");
  CUtensorMap ta, tb;
  int rc = make_fp8_map(&ta, A, M, K, BM);
  if (rc) return rc;
  const bool wide = N % 256 == 0;
  rc = make_fp8_map(&tb, B, N, K, wide ? 256 : 128);
  if (rc) return rc;
  EpiParams ep;
  ep.C = C;
  ep.ldc = ldc;
  ep.M = M;
  ep.N = N;
  ep.bias = static_cast<const uint16_t*>(bias);
  ep.aux = nullptr;
  ep.ld_aux = 0;
  ep.aux_out = nullptr;
  ep.alpha = 1.f;
  ep.beta = 0.f;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint8_t* a_sf = static_cast<const uint8_t*>(sfa);
  const uint8_t* b_sf = static_cast<const uint8_t*>(sfb);
  if (reinterpret_cast<uintptr_t>(C) % 16 == 0) {
    rc = tdb_host::make_tmap_2d(&ep.tmC, C, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, uint64_t(N), uint64_t(M),
                                uint64_t(ldc), 64, 32, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    if (wide)
      return mode == kBias ? mx::launch<256, kTmaBase + kBias>(ta, tb, M, N, K, ep, a_sf, b_sf, s)
                           : mx::launch<256, kTmaBase + kStore>(ta, tb, M, N, K, ep, a_sf, b_sf, s);
    return mode == kBias ? mx::launch<128, kTmaBase + kBias>(ta, tb, M, N, K, ep, a_sf, b_sf, s)
                         : mx::launch<128, kTmaBase + kStore>(ta, tb, M, N, K, ep, a_sf, b_sf, s);
  }
  if (wide)
    return mode == kBias ? mx::launch<256, kBias>(ta, tb, M, N, K, ep, a_sf, b_sf, s)
                         : mx::launch<256, kStore>(ta, tb, M, N, K, ep, a_sf, b_sf, s);
  return mode == kBias ? mx::launch<128, kBias>(ta, tb, M, N, K, ep, a_sf, b_sf, s)
                       : mx::launch<128, kStore>(ta, tb, M, N, K, ep, a_sf, b_sf, s);
}
