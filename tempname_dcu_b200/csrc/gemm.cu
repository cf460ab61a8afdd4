// Plain (single-GPU) tcgen05 GEMM entry point with fused epilogues.
//
// Reference parity: the reference runs every linear layer through
// torch.mm / F.linear (python/flux_dcu/model.py:116,123-124,139-141 and the
// operator chunk GEMM python/flux_dcu/runtime.py:195).  Here those GEMMs are
// one persistent tcgen05 kernel; bias, exact-erf GELU (model.py:261), GELU
// backward, residual adds and fp32 weight-gradient accumulation
// (model.py:401-408) are fused into the epilogue instead of separate kernels.
#include <cmath>
#include <type_traits>

#include "gemm.cuh"
#include "gemm2.cuh"
#include "gemm_epi.cuh"
#include "tensor_map.h"

namespace tdb {
namespace gemm {

template <int BN, bool A_MN, bool B_MN, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int K,
                TileOrder order, const __grid_constant__ EpiParams ep, int* status) {
  typename EpiFor<MODE>::type epi{ep};
  gemm_mainloop<BN, A_MN, B_MN>(&tmA, &tmB, K, order, epi, status);
}

template <int BN, bool A_MN, bool B_MN, int MODE>
static int launch(const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K, const EpiParams& ep,
                  cudaStream_t stream) {
  using Cfg = Config<BN>;
  constexpr int kSmem = Cfg::kSmemBytes + EpiFor<MODE>::type::kSmemBytes;
  auto kern = gemm_kernel<BN, A_MN, B_MN, MODE>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return tdb_host::fail(int(e), "cudaFuncSetAttribute(gemm) failed");
    attr_set[dev & 63] = true;
  }
  TileOrder order;
  order.num_m = (M + BM - 1) / BM;
  order.num_n = (N + BN - 1) / BN;
  order.group_m = 16;
  order.table = nullptr;
  order.num_tiles = order.num_m * order.num_n;
  const int sms = tdb_host::grid_sms();
  const int grid = order.num_tiles < sms ? order.num_tiles : sms;
  kern<<<grid, kThreads, kSmem, stream>>>(ta, tb, K, order, ep, tdb_host::status_ptr());
  tdb_host::launched(1);
  return int(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// 2-CTA (cta_group::2) path: 256 x 256 tiles on SM pairs.
// ---------------------------------------------------------------------------
constexpr int k2Stages = 6;

template <bool A_MN, bool B_MN, int MODE>
__global__ void __launch_bounds__(gemm2::kThreads, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int K,
                 TileOrder order, const __grid_constant__ EpiParams ep, int* status) {
  using Epi = typename EpiFor<MODE>::type;
  Epi epi{ep};
  gemm2::mainloop<A_MN, B_MN, Epi, k2Stages>(&tmA, &tmB, K, order, epi, status);
}

template <bool A_MN, bool B_MN, int MODE>
static int launch2(const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K, const EpiParams& ep,
                   cudaStream_t stream) {
  using Cfg = gemm2::Config<k2Stages>;
  constexpr int kSmem = Cfg::kSmemBytes + EpiFor<MODE>::type::kSmemBytes;
  auto kern = gemm2_kernel<A_MN, B_MN, MODE>;
  static int max_clusters[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(gemm2::kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (!max_clusters[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return tdb_host::fail(int(e), "gemm2: cudaFuncSetAttribute failed");
    cfg.gridDim = dim3(2 * tdb_host::sm_count() / 2);
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    if (e != cudaSuccess || n <= 0) return tdb_host::fail(int(e), "gemm2: no active 2-CTA clusters possible");
    max_clusters[dev & 63] = n;
  }
  TileOrder order;
  order.num_m = (M + 255) / 256;
  order.num_n = (N + 255) / 256;
  order.group_m = 8;
  order.table = nullptr;
  order.num_tiles = order.num_m * order.num_n;
  int clusters = order.num_tiles < max_clusters[dev & 63] ? order.num_tiles : max_clusters[dev & 63];
  if (clusters > tdb_host::grid_sms() / 2) clusters = tdb_host::grid_sms() / 2 > 0 ? tdb_host::grid_sms() / 2 : 1;
  cfg.gridDim = dim3(2 * clusters);
  int* status = tdb_host::status_ptr();
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, K, order, ep, status);
  tdb_host::launched(1);
  if (e != cudaSuccess) return tdb_host::fail(int(e), "gemm2: launch failed");
  return 0;
}

template <bool A_MN, bool B_MN>
static int dispatch2(int mode, const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K,
                     const EpiParams& ep, cudaStream_t s) {
  switch (mode) {
    case kStore: return launch2<A_MN, B_MN, kStore>(ta, tb, M, N, K, ep, s);
    case kBias: return launch2<A_MN, B_MN, kBias>(ta, tb, M, N, K, ep, s);
    case kBiasGelu: return launch2<A_MN, B_MN, kBiasGelu>(ta, tb, M, N, K, ep, s);
    case kGeluBwd: return launch2<A_MN, B_MN, kGeluBwd>(ta, tb, M, N, K, ep, s);
    case kAccF32: return launch2<A_MN, B_MN, kAccF32>(ta, tb, M, N, K, ep, s);
    case kAccF32Tma: return launch2<A_MN, B_MN, kAccF32Tma>(ta, tb, M, N, K, ep, s);
    case kTmaBase + 0: return launch2<A_MN, B_MN, kTmaBase + 0>(ta, tb, M, N, K, ep, s);
    case kTmaBase + 1: return launch2<A_MN, B_MN, kTmaBase + 1>(ta, tb, M, N, K, ep, s);
    case kTmaBase + 2: return launch2<A_MN, B_MN, kTmaBase + 2>(ta, tb, M, N, K, ep, s);
    case kTmaBase + 3: return launch2<A_MN, B_MN, kTmaBase + 3>(ta, tb, M, N, K, ep, s);
    case kTmaBase + 5: return launch2<A_MN, B_MN, kTmaBase + 5>(ta, tb, M, N, K, ep, s);
    case kBiasResidual: return launch2<A_MN, B_MN, kBiasResidual>(ta, tb, M, N, K, ep, s);
  }
  return tdb_host::fail(int(cudaErrorInvalidValue), "unknown epilogue mode %d", mode);
}

template <int BN, bool A_MN, bool B_MN>
static int dispatch_mode(int mode, const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K,
                         const EpiParams& ep, cudaStream_t s) {
  switch (mode) {
    case kStore: return launch<BN, A_MN, B_MN, kStore>(ta, tb, M, N, K, ep, s);
    case kBias: return launch<BN, A_MN, B_MN, kBias>(ta, tb, M, N, K, ep, s);
    case kBiasGelu: return launch<BN, A_MN, B_MN, kBiasGelu>(ta, tb, M, N, K, ep, s);
    case kGeluBwd: return launch<BN, A_MN, B_MN, kGeluBwd>(ta, tb, M, N, K, ep, s);
    case kAccF32: return launch<BN, A_MN, B_MN, kAccF32>(ta, tb, M, N, K, ep, s);
    case kAccF32Tma: return launch<BN, A_MN, B_MN, kAccF32Tma>(ta, tb, M, N, K, ep, s);
    case kTmaBase + 0: return launch<BN, A_MN, B_MN, kTmaBase + 0>(ta, tb, M, N, K, ep, s);
    case kTmaBase + 1: return launch<BN, A_MN, B_MN, kTmaBase + 1>(ta, tb, M, N, K, ep, s);
    case kTmaBase + 2: return launch<BN, A_MN, B_MN, kTmaBase + 2>(ta, tb, M, N, K, ep, s);
    case kTmaBase + 3: return launch<BN, A_MN, B_MN, kTmaBase + 3>(ta, tb, M, N, K, ep, s);
    case kTmaBase + 5: return launch<BN, A_MN, B_MN, kTmaBase + 5>(ta, tb, M, N, K, ep, s);
    case kBiasResidual: return launch<BN, A_MN, B_MN, kBiasResidual>(ta, tb, M, N, K, ep, s);
  }
  return tdb_host::fail(int(cudaErrorInvalidValue), "unknown epilogue mode %d", mode);
}

template <int BN>
static int dispatch_major(int a_mn, int b_mn, int mode, const CUtensorMap& ta, const CUtensorMap& tb, int M, int N,
                          int K, const EpiParams& ep, cudaStream_t s) {
  if (!a_mn && !b_mn) return dispatch_mode<BN, false, false>(mode, ta, tb, M, N, K, ep, s);
  if (!a_mn && b_mn) return dispatch_mode<BN, false, true>(mode, ta, tb, M, N, K, ep, s);
  if (a_mn && b_mn) return dispatch_mode<BN, true, true>(mode, ta, tb, M, N, K, ep, s);
  return dispatch_mode<BN, true, false>(mode, ta, tb, M, N, K, ep, s);
}

// Builds the TMA map of one operand.  K-major: rows = mn extent, inner = K,
// box {64, tile_mn}.  MN-major: rows = K, inner = mn extent, box {64, 64}.
int make_operand_map(CUtensorMap* map, const void* ptr, bool mn_major, int mn, int K, int64_t ld, int tile_mn) {
  if (!mn_major)
    return tdb_host::make_tmap_2d(map, ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, uint64_t(K), uint64_t(mn),
                                  uint64_t(ld), BK, uint32_t(tile_mn), CU_TENSOR_MAP_SWIZZLE_128B);
  return tdb_host::make_tmap_2d(map, ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, uint64_t(mn), uint64_t(K),
                                uint64_t(ld), 64, BK, CU_TENSOR_MAP_SWIZZLE_128B);
}

// Tile shape for an M x N output: the candidate with the best product of
// (a) wave efficiency -- work units over the units the machine runs in
// ceil(units / slots) full waves (2-CTA tiles occupy SM pairs), (b) the useful
// fraction of partial edge tiles and (c) a per-shape throughput factor (larger
// tiles re-read less shared memory per MMA).  Returns the bn code of tdb_gemm.
int pick_tile(int M, int N, int K, int sms) {
  struct Cand {
    int code, tm, tn, slots;
    double speed;
  };
  const Cand cands[4] = {{512, 256, 256, sms / 2, 1.00}, {256, 128, 256, sms, 0.95}, {192, 128, 192, sms, 0.92},
                         {128, 128, 128, sms, 0.85}};
  int best = 128;
  double best_score = -1.0;
  for (const Cand& c : cands) {
    if (c.code == 512 && (M < 256 || N < 256 || K < 256)) continue;
    if (N <= 128 && c.tn > 128) continue;
    const double tiles_m = double((M + c.tm - 1) / c.tm), tiles_n = double((N + c.tn - 1) / c.tn);
    const double units = tiles_m * tiles_n;
    const double waves = std::ceil(units / c.slots);
    const double useful = (double(M) / c.tm) * (double(N) / c.tn) / units;
    const double score = units / (waves * c.slots) * useful * c.speed;
    if (score > best_score + 1e-9) {
      best_score = score;
      best = c.code;
    }
  }
  return best;
}

}  // namespace gemm
}  // namespace tdb

using namespace tdb;
using namespace tdb::gemm;

// Tile choice of tdb_gemm for a shape on a GPU with `sms` SMs (bn code: 128,
// 192, 256, or 512 = 2-CTA 256 x 256).  Pure function of its arguments.
TDB_API int tdb_gemm_pick_tile(int M, int N, int K, int sms) { return tdb::gemm::pick_tile(M, N, K, sms); }

// C = epilogue(A * B^T).  a_mn / b_mn select the storage of A ([M,K] vs [K,M])
// and B ([N,K] vs [K,N]); lda / ldb are the row strides of that storage in
// elements.  C is bf16 [M, ldc] except for mode 4 (fp32).  bn = 0 picks the
// tile width automatically (256 unless that leaves SMs idle).
TDB_API int tdb_gemm(const void* A, int a_mn, int64_t lda, const void* B, int b_mn, int64_t ldb, void* C,
                     int64_t ldc, int M, int N, int K, int mode, const void* bias, const void* aux, int64_t ld_aux,
                     void* aux_out, float alpha, float beta, int bn, void* stream) {
  if (!A || !B || !C || M <= 0 || N <= 0 || K <= 0 || mode < kStore || mode > kBiasResidual)
    return tdb_host::fail(int(cudaErrorInvalidValue), "gemm: bad pointers, sizes or mode");
  if (K % 8 || (a_mn && M % 8) || (b_mn && N % 8) || N % 8 || ldc % 8)
    return tdb_host::fail(int(cudaErrorInvalidValue), "gemm: K, N, ldc (and M / N for MN-major) must be multiples of 8");
  if ((mode == kBiasGelu && (!aux_out || ld_aux % 8)) || ((mode == kGeluBwd || mode == kBiasResidual) && (!aux || ld_aux % 8)))
    return tdb_host::fail(int(cudaErrorInvalidValue), "gemm: epilogue mode %d needs an aligned aux tensor", mode);
  if (bias && (reinterpret_cast<uintptr_t>(bias) % 16))
    return tdb_host::fail(int(cudaErrorInvalidValue), "gemm: bias must be 16-byte aligned");
  if (bn == 0) bn = pick_tile(M, N, K, tdb_host::sm_count());
  if (bn != 128 && bn != 192 && bn != 256 && bn != 512)
    return tdb_host::fail(int(cudaErrorInvalidValue), "gemm: bn must be 128, 192, 256 or 512 (2-CTA)");
  CUtensorMap ta, tb;
  int rc = make_operand_map(&ta, A, a_mn, M, K, lda, BM);
  if (rc) return rc;
  rc = make_operand_map(&tb, B, b_mn, N, K, ldb, bn == 512 ? 128 : bn);
  if (rc) return rc;
  EpiParams ep;
  ep.C = C;
  ep.ldc = ldc;
  ep.M = M;
  ep.N = N;
  ep.bias = static_cast<const uint16_t*>(bias);
  ep.aux = static_cast<const uint16_t*>(aux);
  ep.ld_aux = ld_aux;
  ep.aux_out = static_cast<uint16_t*>(aux_out);
  ep.alpha = alpha;
  ep.beta = beta;
  if (mode == kAccF32 && (beta == 0.f || beta == 1.f) && reinterpret_cast<uintptr_t>(C) % 16 == 0 && ldc % 4 == 0) {
    rc = tdb_host::make_tmap_2d(&ep.tmC, C, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, uint64_t(N), uint64_t(M),
                                uint64_t(ldc), 32, 32, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    mode = kAccF32Tma;
  } else if (mode != kAccF32 && reinterpret_cast<uintptr_t>(C) % 16 == 0 &&
             (mode != kBiasGelu || reinterpret_cast<uintptr_t>(aux_out) % 16 == 0)) {
    rc = tdb_host::make_tmap_2d(&ep.tmC, C, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, uint64_t(N), uint64_t(M),
                                uint64_t(ldc), 64, 32, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    if (mode == kBiasGelu) {
      rc = tdb_host::make_tmap_2d(&ep.tmAux, aux_out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, uint64_t(N), uint64_t(M),
                                  uint64_t(ld_aux), 64, 32, CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc) return rc;
    }
    mode += kTmaBase;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (bn == 512) {
    if (!a_mn && !b_mn) return dispatch2<false, false>(mode, ta, tb, M, N, K, ep, s);
    if (!a_mn && b_mn) return dispatch2<false, true>(mode, ta, tb, M, N, K, ep, s);
    if (a_mn && b_mn) return dispatch2<true, true>(mode, ta, tb, M, N, K, ep, s);
    return dispatch2<true, false>(mode, ta, tb, M, N, K, ep, s);
  }
  if (bn == 256) return dispatch_major<256>(a_mn, b_mn, mode, ta, tb, M, N, K, ep, s);
  if (bn == 192) return dispatch_major<192>(a_mn, b_mn, mode, ta, tb, M, N, K, ep, s);
  return dispatch_major<128>(a_mn, b_mn, mode, ta, tb, M, N, K, ep, s);
}
